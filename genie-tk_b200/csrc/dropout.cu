// Training-mode channel dropout of the residual updates (reference
// src/genie_tk/pair_transform.py:26-61, applied at :182-189 as p = p + dropout(update)).
// DropoutRowwise draws one mask [B, 1, N, C] shared by every row i, DropoutColumnwise one
// mask [B, N, 1, C] shared by every column j. The residual epilogues (K2e, K4e) take such a
// mask as keep bits, B * N vectors of ceil(C / 128) groups of 128 bits (generated and packed
// here as that many 128-bit vectors), and apply it while they add the residual,
// so the masked update is never written out. This file makes the bit vectors:
//   dropout_philox_kernel  from a counter-based generator, Philox4x32-10 (Salmon, Moraes,
//                          Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11):
//                          channel c of vector v keeps when output word c % 4 of
//                          Philox(counter = (v * 32 + c / 4, offset), key = seed) is at least
//                          floor(p * 2^32);
//   dropout_pack_kernel    from a multiplier tensor [n][128] (0 = dropped), which is how the
//                          Python layer packs the mask drawn by nn.Dropout itself, so that a
//                          seeded run consumes the random stream exactly as the reference does.
#include <cuda_runtime.h>

#include <cmath>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {

namespace philox {
// The Philox-4x32 multipliers and Weyl key increments of the SC'11 paper.
constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
}  // namespace philox

// Ten rounds of Philox-4x32 on `ctr` with key `key` (the key is bumped between rounds).
__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    if (round > 0) {
      k0 += philox::kW0;
      k1 += philox::kW1;
    }
    const uint32_t lo0 = philox::kM0 * ctr.x, hi0 = __umulhi(philox::kM0, ctr.x);
    const uint32_t lo1 = philox::kM1 * ctr.z, hi1 = __umulhi(philox::kM1, ctr.z);
    ctr = make_uint4(hi1 ^ ctr.y ^ k0, lo1, hi0 ^ ctr.w ^ k1, lo0);
  }
  return ctr;
}

// One thread per 32-bit keep word (channels 32 w .. 32 w + 31 of vector v): 8 Philox blocks.
__global__ void __launch_bounds__(256)
    dropout_philox_kernel(uint64_t seed, uint64_t offset, uint32_t threshold, int64_t n_words,
                          uint32_t* __restrict__ keep) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n_words; t += stride) {
    const int64_t v = t >> 2;
    const int w = static_cast<int>(t & 3);
    uint32_t bits = 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint64_t block = static_cast<uint64_t>(v) * 32u + static_cast<uint64_t>(w * 8 + g);
      const uint4 r = philox4x32_10(make_uint4(static_cast<uint32_t>(block), static_cast<uint32_t>(block >> 32),
                                               static_cast<uint32_t>(offset), static_cast<uint32_t>(offset >> 32)),
                                    static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
      bits |= static_cast<uint32_t>(r.x >= threshold) << (g * 4 + 0);
      bits |= static_cast<uint32_t>(r.y >= threshold) << (g * 4 + 1);
      bits |= static_cast<uint32_t>(r.z >= threshold) << (g * 4 + 2);
      bits |= static_cast<uint32_t>(r.w >= threshold) << (g * 4 + 3);
    }
    keep[t] = bits;
  }
}

// One warp per 32-bit keep word: lane l reads multiplier 32 w + l of its vector, the
// ballot is the word.
__global__ void __launch_bounds__(256)
    dropout_pack_kernel(const float* __restrict__ mult, int64_t n_words, uint32_t* __restrict__ keep) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; t < n_words; t += nwarps) {
    const float m = __ldg(mult + t * 32 + lane);
    const uint32_t bits = __ballot_sync(0xffffffffu, m != 0.f);
    if (lane == 0) keep[t] = bits;
  }
}

int drop_args(const gtk_dropout* d, int64_t B, int64_t N, bool transposed, int channels, DropArgs* out) {
  *out = DropArgs{};
  if (!d) return GTK_OK;  // no dropout
  if (!d->keep_bits) return fail(GTK_ERR_INVALID_ARG, "dropout: keep_bits is NULL");
  if (reinterpret_cast<uintptr_t>(d->keep_bits) & 15)
    return fail(GTK_ERR_ALIGNMENT, "dropout: keep_bits must be 16-byte aligned");
  if (!std::isfinite(d->scale) || d->scale < 0.f) return fail(GTK_ERR_INVALID_ARG, "dropout: bad scale");
  if (B < 1 || N < 1) return fail(GTK_ERR_INVALID_ARG, "dropout: bad B/N");
  out->keep = reinterpret_cast<const uint4*>(d->keep_bits);
  out->scale = d->scale;
  // DropoutRowwise's vector is the pair's column j, DropoutColumnwise's its row i; in a
  // transposed kernel frame (rows = j) the two swap.
  out->by_row = ((d->shared_across_rows != 0) == transposed) ? 1 : 0;
  out->ld = N;
  out->groups = (channels + 127) / 128;
  return GTK_OK;
}

static int grid_for(int64_t work_items, int per_block) {
  const int64_t need = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  return static_cast<int>(need < 1 ? 1 : (need < cap ? need : cap));
}

}  // namespace gtk

using namespace gtk;

extern "C" {

int gtk_dropout_keep_bits_philox(uint64_t seed, uint64_t offset, double p, int64_t n_vectors, uint32_t* keep_bits,
                                 void* stream) {
  if (!(p >= 0.0 && p < 1.0)) return fail(GTK_ERR_INVALID_ARG, "dropout: p must be in [0, 1)");
  if (!dims_ok(n_vectors, int64_t(1) << 40)) return fail(GTK_ERR_INVALID_ARG, "dropout: bad n_vectors");
  if (int e = check_ptr(keep_bits, "keep_bits")) return e;
  if (int e = check_device()) return e;
  const double t = std::floor(p * 4294967296.0);
  const uint32_t threshold = t >= 4294967295.0 ? 0xFFFFFFFFu : static_cast<uint32_t>(t);
  const int64_t n_words = n_vectors * 4;
  dropout_philox_kernel<<<grid_for(n_words, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      seed, offset, threshold, n_words, keep_bits);
  return check_launch("dropout_philox_kernel");
}

int gtk_dropout_pack_keep_bits(const float* multipliers, int64_t n_vectors, uint32_t* keep_bits, void* stream) {
  if (!dims_ok(n_vectors, int64_t(1) << 40)) return fail(GTK_ERR_INVALID_ARG, "dropout: bad n_vectors");
  if (int e = check_ptr(multipliers, "multipliers", 4)) return e;
  if (int e = check_ptr(keep_bits, "keep_bits")) return e;
  if (int e = check_device()) return e;
  const int64_t n_words = n_vectors * 4;
  dropout_pack_kernel<<<grid_for(n_words * 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      multipliers, n_words, keep_bits);
  return check_launch("dropout_pack_kernel");
}

}  // extern "C"
