// Pair transition (reference src/genie_tk/pair_transform.py:64-84: LayerNorm -> Linear(c_p, 4 c_p)
// -> ReLU -> Linear(4 c_p, c_p)), with the pair transform layer's residual and final mask
// (pair_transform.py:190-193: p = p + transition(p); p = p * p_mask) folded into the last
// kernel. Two persistent kernels, both HBM-bound:
//
//  K5a transition_in_kernel   LN (affine folded into W1 / b1) + the 128 -> 512 projection
//                             (one 128 x 512 x 128 tcgen05 GEMM per 128-pair tile, two TMEM
//                             halves) + bias + ReLU -> hidden rows h fp16 [pairs][512].
//  K5b transition_out_kernel  h W2^T (K = 512 through a two-stage TMA ring, W2 resident)
//                             + b2 (+ residual z) (* mask) -> fp32 pairs, residual and
//                             output through a TMA slab ring.
//
// A single fused kernel does not fit: W1 and W2 are 128 KB each in fp16 and a 128-pair
// tile needs its 64 KB z block and a 32 KB operand besides, so one of the weights would be
// re-streamed from L2 for every tile (256 KB per 128 pairs). The hidden rows cost 2 KB per
// pair of HBM traffic instead (written once, read once); the whole transition moves
// ~3.6 KB per pair against ~12 KB for the unfused PyTorch ops.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"
#include "general.h"

namespace gtk {

// ----------------------------------------------------------------------------------
// Packed weights:
//   W1  fp16 [512][128]  linear_1.weight * gamma (LayerNorm scale folded; [out, in] =
//                        K-major B operand)
//   W2  fp16 [128][512]  linear_2.weight ([out, in], K = 512 contiguous)
//   vec fp32: b1[512] = linear_1.bias + W1 beta, b2[128] = linear_2.bias
// LN(x) W1^T + b1 = xhat (W1 gamma)^T + (W1 beta + b1), so K5a's producers write
// xhat = (x - mu) * rstd alone.
// ----------------------------------------------------------------------------------
namespace tnpack {
constexpr int kCp = 128, kHid = 512;
constexpr size_t kW1 = 0;
constexpr size_t kW2 = size_t(kHid) * kCp * 2;
constexpr size_t kVec = kW2 + size_t(kCp) * kHid * 2;
constexpr int kVB1 = 0, kVB2 = 512, kVecFloats = 640;
constexpr size_t kBytes = kVec + kVecFloats * 4;
}  // namespace tnpack

// Packs a transition of expansion n <= 4 (hidden = 128 n) into the tuned 512-unit layout:
// hidden units past 128 n have zero W1 rows and b1, so ReLU makes them exactly 0, and zero W2
// columns, so the result is the n-unit transition's.
__global__ void transition_pack_kernel(gtk_transition_params p, uint8_t* packed, int hid) {
  using namespace tnpack;
  __half* w1 = reinterpret_cast<__half*>(packed + kW1);
  __half* w2 = reinterpret_cast<__half*>(packed + kW2);
  float* vec = reinterpret_cast<float*>(packed + kVec);
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nthreads = gridDim.x * blockDim.x;
  for (int e = tid; e < kHid * kCp; e += nthreads) {
    const int r = e / kCp, c = e % kCp;
    w1[e] = f16_sat(r < hid ? p.w1[e] * p.ln_w[c] : 0.f);
  }
  for (int e = tid; e < kCp * kHid; e += nthreads) {
    const int o = e / kHid, r = e % kHid;
    w2[e] = f16_sat(r < hid ? p.w2[o * hid + r] : 0.f);
  }
  for (int r = tid; r < kHid; r += nthreads) {
    float acc = 0.f;
    if (r < hid) {
      acc = p.b1 ? p.b1[r] : 0.f;
      for (int c = 0; c < kCp; ++c) acc += p.w1[r * kCp + c] * p.ln_b[c];
    }
    vec[kVB1 + r] = acc;
  }
  for (int r = tid; r < kCp; r += nthreads) vec[kVB2 + r] = p.b2 ? p.b2[r] : 0.f;
}

// ----------------------------------------------------------------------------------
// K5a: persistent LN + 128 -> 512 projection + bias + ReLU. Tile = 128 consecutive pairs
// (b, i, j0..j0+127). 512 threads, the organisation of the attention projection kernel:
//   warps 0-7  LayerNorm producers, two threads per pair row (64 channels each, statistics
//              combined with one shuffle): one pass reads the staged 128-B-swizzled z tile
//              into registers and releases it, then writes xhat as the fp16 operand A.
//              Thread 0 is also the TMA producer (W1 once, the z tiles) and MMA issuer.
//   warps 8-15 epilogue, thread = pair (TMEM lane quarter = warp % 4); warps 8-11 take
//              hidden units 0-127 of each TMEM half, warps 12-15 units 128-255, in 16-column
//              chunks whose TMEM loads run one chunk ahead: + b1, ReLU, fp16, one 32-byte
//              store per chunk into the pair's 1 KB hidden row.
// TMEM: half 0 = hidden 0-255 (columns 0-255), half 1 = hidden 256-511; the epilogue of
// half 0 overlaps the MMAs of half 1, the next tile's LayerNorm and z load overlap both.
// Shared memory: W1 128 KB | z 64 KB | A 32 KB | b1 2 KB | barriers (no alignment slack:
// the kernel checks for a 1024-aligned dynamic shared-memory base).
// ----------------------------------------------------------------------------------
namespace k5a {
constexpr int kThreads = 512;
constexpr uint32_t kW = 0, kZ = 131072, kA = 196608, kB1 = 229376, kBar = kB1 + 2048;
constexpr uint32_t kSmem = kBar + 128;
static_assert(kSmem <= 232448, "K5a shared memory");
}  // namespace k5a

struct K5aBars {
  uint64_t wbar;
  uint64_t z_full, z_empty;
  uint64_t a_full, a_empty;
  uint64_t d_full[2], d_empty[2];
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K5aBars) <= 128, "K5a barrier block");

__global__ void __launch_bounds__(k5a::kThreads, 1)
    transition_in_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap z_map,
                         const float* __restrict__ vec, __half* __restrict__ hid, int N, int rows, int n_jt,
                         int n_tiles, uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t dsmem[];
  if (smem_u32(dsmem) & 1023u) {  // uniform across the CTA: every thread leaves here
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadLaunch);
    return;
  }
  uint8_t* smem = dsmem;
  K5aBars* bars = reinterpret_cast<K5aBars*>(smem + k5a::kBar);
  CtaGuard* guard = &bars->guard;
  float* b1_s = reinterpret_cast<float*>(smem + k5a::kB1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(&bars->wbar, 1);
    mbar_init(&bars->z_full, 1);
    mbar_init(&bars->z_empty, 256);
    mbar_init(&bars->a_full, 256);
    mbar_init(&bars->a_empty, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->d_full[x], 1);
      mbar_init(&bars->d_empty[x], 256);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  b1_s[tid] = vec[tnpack::kVB1 + tid];  // 512 threads, 512 biases
  if (warp == 8) {
    tmem_alloc(&bars->tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;

  if (warp < 8) {
    // ------- LayerNorm producers (two threads per pair row); thread 0 also issues -------
    const int p = warp * 16 + (lane >> 1), half = lane & 1;
    auto load_z = [&](int tile) {
      const int jt = tile % n_jt, rb = tile / n_jt;
      const int r = rb % rows, b = rb / rows;
      mbar_arrive_expect_tx(&bars->z_full, 65536);
#pragma unroll
      for (int q = 0; q < 4; ++q) tma_load_4d(smem + k5a::kZ + q * 16384, &z_map, &bars->z_full, q * 32, jt * 128, r, b);
    };
    int loaded = 0;  // z tiles requested (thread 0)
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars->wbar, 131072);
#pragma unroll
      for (int kh = 0; kh < 2; ++kh)
#pragma unroll
        for (int rb = 0; rb < 4; ++rb)
          tma_load_2d(smem + k5a::kW + kh * 65536 + rb * 16384, &w_map, &bars->wbar, kh * 64, rb * 128);
      load_z(blockIdx.x);  // the grid never exceeds the tile count
      loaded = 1;
    }
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->z_full, it & 1, guard, status, kStatusTimeoutProducer));
      if (!ok) break;
      float v[64];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float4 t = lds_f4(smem + k5a::kZ + (2 * half + q) * 16384 + swz128(p, ch));
          v[q * 32 + ch * 4 + 0] = t.x;
          v[q * 32 + ch * 4 + 1] = t.y;
          v[q * 32 + ch * 4 + 2] = t.z;
          v[q * 32 + ch * 4 + 3] = t.w;
        }
      // the z tile may be refilled once every loaded value has been consumed (see
      // mbar_arrive_after): the local sum reads all 64 of them
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) s4[c & 3] += v[c];
      float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      mbar_arrive_after(&bars->z_empty, sum);
      if (warp == 0) {
        // thread 0: refill z with the next tile once every producer has read this one
        bool w = true;
        if (lane == 0 && tile + static_cast<int>(gridDim.x) < n_tiles) {
          w = mbar_wait(&bars->z_empty, it & 1, guard, status, kStatusTimeoutMma);
          if (w) {
            load_z(tile + gridDim.x);
            ++loaded;
          }
        }
        ok = __all_sync(0xffffffffu, w);
        if (!ok) break;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      const float mean = sum * (1.f / 128.f);
      float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float d = v[c] - mean;
        q4[c & 3] += d * d;
      }
      float ss = (q4[0] + q4[1]) + (q4[2] + q4[3]);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rstd = rsqrtf(ss * (1.f / 128.f) + 1e-5f);
      ok = it < 1 || __all_sync(0xffffffffu, mbar_wait(&bars->a_empty, (it - 1) & 1, guard, status,
                                                      kStatusTimeoutProducer));
      if (!ok) break;
      // xhat only: gamma and beta are folded into W1 and b1
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int c = ch * 8;
        uint4 o;
        o.x = pack_f16x2((v[c + 0] - mean) * rstd, (v[c + 1] - mean) * rstd);
        o.y = pack_f16x2((v[c + 2] - mean) * rstd, (v[c + 3] - mean) * rstd);
        o.z = pack_f16x2((v[c + 4] - mean) * rstd, (v[c + 5] - mean) * rstd);
        o.w = pack_f16x2((v[c + 6] - mean) * rstd, (v[c + 7] - mean) * rstd);
        sts_u4(smem + k5a::kA + half * 16384 + swz128(p, ch), o);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->a_full);
      if (warp == 0) {
        // thread 0: the tile's MMAs, half h once the epilogue has drained half h of the
        // previous tile
        bool mw = true;
        if (lane == 0) {
          const uint32_t idesc = make_idesc_f16(128, 256, 0, 0);
          const uint32_t w0 = smem_u32(smem + k5a::kW), a0 = smem_u32(smem + k5a::kA);
          mw = mbar_wait(&bars->a_full, it & 1, guard, status, kStatusTimeoutMma);
          if (mw && it == 0) mw = mbar_wait(&bars->wbar, 0, guard, status, kStatusTimeoutMma);
          for (int h = 0; mw && h < 2; ++h) {
            if (it >= 1) mw = mbar_wait(&bars->d_empty[h], (it - 1) & 1, guard, status, kStatusTimeoutMma);
            if (!mw) break;
            tc_fence_after();
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const int kh = ks >> 2, kin = ks & 3;
              umma_ss(tmem + h * 256, make_sdesc(a0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128),
                      make_sdesc(w0 + kh * 65536 + h * 32768 + kin * 32, 16, 1024, Swz::k128), idesc, ks > 0 ? 1u : 0u);
            }
            umma_commit(&bars->d_full[h]);
          }
          if (mw) umma_commit(&bars->a_empty);
        }
        ok = __all_sync(0xffffffffu, mw);
        if (!ok) break;
      }
    }
    if (!ok && tid == 0) {
      // abort: wait (bounded) for this thread's MMAs and TMA loads still in flight
      umma_commit(&bars->drain);
      mbar_wait_drain(&bars->drain, 0);
      if (loaded > 0) mbar_wait_drain(&bars->z_full, (loaded - 1) & 1);
      mbar_wait_drain(&bars->wbar, 0);
    }
  } else {
    // ---------- epilogue: thread = pair; hidden units 128 hh .. +127 of each TMEM half ----------
    const int q4 = warp & 3, hh = (warp - 8) >> 2;
    const int p = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t sat = 0;  // a hidden value beyond the fp16 range was clamped
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int jt = tile % n_jt, rb = tile / n_jt;
      const int j = jt * 128 + p;
      const bool valid = j < N;
      __half* hrow = hid + (static_cast<size_t>(rb) * N + j) * tnpack::kHid;
      bool ok = true;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[h], it & 1, guard, status, kStatusTimeoutConsumer));
        if (!ok) break;
        tc_fence_after();
        const int u0 = h * 256 + hh * 128;  // first hidden unit of this thread's range
        const uint32_t tb = tmem + lane_off + u0;
        uint32_t x[2][16];
        tmem_ld16(tb, x[0]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int cur = k & 1;
          tmem_wait_ld_regs(x[cur]);
          if (k + 1 < 8) tmem_ld16(tb + (k + 1) * 16, x[cur ^ 1]);
          if (valid) {
            uint32_t w[8];
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              const float4 bb = *reinterpret_cast<const float4*>(b1_s + u0 + k * 16 + e4 * 4);
              w[2 * e4] = pack_f16x2_chk(fmaxf(__uint_as_float(x[cur][e4 * 4 + 0]) + bb.x, 0.f),
                                         fmaxf(__uint_as_float(x[cur][e4 * 4 + 1]) + bb.y, 0.f), sat);
              w[2 * e4 + 1] = pack_f16x2_chk(fmaxf(__uint_as_float(x[cur][e4 * 4 + 2]) + bb.z, 0.f),
                                             fmaxf(__uint_as_float(x[cur][e4 * 4 + 3]) + bb.w, 0.f), sat);
            }
            stg_v8(hrow + u0 + k * 16, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]);
          }
        }
        tc_fence_before();
        mbar_arrive(&bars->d_empty[h]);
      }
      if (!ok) break;
    }
    flag_saturation(sat, status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------------
// K5b: persistent out = (h W2^T + b2 [+ z]) [* mask]. Tile = 128 pairs; the 128 x 512
// fp16 hidden rows arrive as four 32 KB K-chunks through a two-stage TMA ring while W2
// (128 KB) stays resident; one tile's accumulator is 128 TMEM columns, double buffered.
// The output is four 32-channel fp32 slabs through a two-buffer ring: the slab manager
// loads the residual slab of z, the epilogue adds accumulator, bias (and applies the mask)
// in place, and the slab manager stores it. 224 threads:
//   warps 0-3  epilogue: thread = pair (TMEM lane);
//   warp 4     lane 0: TMA producer (W2 once, the hidden K-chunks);
//   warp 5     lane 0: TMEM allocator and MMA issuer;
//   warp 6     lane 0: slab manager (residual loads, output stores).
// Shared memory: W2 128 KB | hidden ring 2 x 32 KB | slabs 2 x 16 KB | b2 | barriers
// (no alignment slack; checked as in K5a).
// ----------------------------------------------------------------------------------
namespace k5b {
constexpr int kThreads = 224;
constexpr int kStages = 2, kSlabs = 2;
constexpr uint32_t kW = 0, kA = 131072, kO = kA + kStages * 32768, kVec = kO + kSlabs * 16384, kBar = kVec + 512;
constexpr uint32_t kSmem = kBar + 256;
static_assert(kSmem <= 232448, "K5b shared memory");
}  // namespace k5b

struct K5bBars {
  uint64_t wbar;
  uint64_t a_full[k5b::kStages], a_empty[k5b::kStages];
  uint64_t d_full[2], d_empty[2];
  uint64_t o_full[k5b::kSlabs];
  uint64_t slab_ready[k5b::kSlabs];  // 128 epilogue threads wrote the slab
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K5bBars) <= 256, "K5b barrier block");

__global__ void __launch_bounds__(k5b::kThreads, 1)
    transition_out_kernel(const __grid_constant__ CUtensorMap h_map, const __grid_constant__ CUtensorMap w_map,
                          const __grid_constant__ CUtensorMap z_map, const __grid_constant__ CUtensorMap out_map,
                          const float* __restrict__ vec, const float* __restrict__ mask, int N, int rows,
                          int add_residual, int n_jt, int n_tiles, uint32_t* status) {
  using namespace k5b;
  extern __shared__ __align__(1024) uint8_t dsmem[];
  if (smem_u32(dsmem) & 1023u) {  // uniform across the CTA: every thread leaves here
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadLaunch);
    return;
  }
  uint8_t* smem = dsmem;
  K5bBars* bars = reinterpret_cast<K5bBars*>(smem + kBar);
  CtaGuard* guard = &bars->guard;
  float* sb2 = reinterpret_cast<float*>(smem + kVec);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(&bars->wbar, 1);
    for (int x = 0; x < kStages; ++x) {
      mbar_init(&bars->a_full[x], 1);
      mbar_init(&bars->a_empty[x], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->d_full[x], 1);
      mbar_init(&bars->d_empty[x], 128);
    }
    for (int x = 0; x < kSlabs; ++x) {
      mbar_init(&bars->o_full[x], 1);
      mbar_init(&bars->slab_ready[x], 128);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (tid < 128) sb2[tid] = vec[tnpack::kVB2 + tid];
  if (warp == 5) {
    tmem_alloc(&bars->tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;
  const int n_mine = (n_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                     static_cast<int>(gridDim.x);

  if (warp == 4) {
    // ------------------ TMA producer: W2 once, then the hidden K-chunks ------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->wbar, 131072);
#pragma unroll
      for (int kb = 0; kb < 8; ++kb) tma_load_2d(smem + kW + kb * 16384, &w_map, &bars->wbar, kb * 64, 0);
      bool ok = true;
      const int total = 4 * n_mine;
      int q = 0;
      for (; q < total; ++q) {
        const int st = q % kStages, c = q & 3;
        const int tile = blockIdx.x + (q >> 2) * gridDim.x;
        const int jt = tile % n_jt, rb = tile / n_jt;
        if (q >= kStages &&
            !mbar_wait(&bars->a_empty[st], ((q / kStages) - 1) & 1, guard, status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->a_full[st], 32768);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
          tma_load_3d(smem + kA + st * 32768 + kh * 16384, &h_map, &bars->a_full[st], c * 128 + kh * 64, jt * 128, rb);
      }
      if (!ok)
        for (int t = (q > kStages ? q - kStages : 0); t < q; ++t)
          mbar_wait_drain(&bars->a_full[t % kStages], (t / kStages) & 1);
      mbar_wait_drain(&bars->wbar, 0);
    }
  } else if (warp == 5) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(&bars->wbar, 0, guard, status, kStatusTimeoutMma);
      const uint32_t idesc = make_idesc_f16(128, 128, 0, 0);
      const uint32_t w0 = smem_u32(smem + kW), a0 = smem_u32(smem + kA);
      int q = 0;
      for (int it = 0; ok && it < n_mine; ++it) {
        const int s = it & 1;
        if (it >= 2) ok = mbar_wait(&bars->d_empty[s], ((it >> 1) - 1) & 1, guard, status, kStatusTimeoutMma);
        for (int c = 0; ok && c < 4; ++c, ++q) {
          const int st = q % kStages;
          ok = mbar_wait(&bars->a_full[st], (q / kStages) & 1, guard, status, kStatusTimeoutMma);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const int kh = ks >> 2, kin = ks & 3;
            umma_ss(tmem + s * 128, make_sdesc(a0 + st * 32768 + kh * 16384 + kin * 32, 16, 1024, Swz::k128),
                    make_sdesc(w0 + (2 * c + kh) * 16384 + kin * 32, 16, 1024, Swz::k128), idesc,
                    (c > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&bars->a_empty[st]);
        }
        if (ok) umma_commit(&bars->d_full[s]);
      }
      if (!ok) {
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else if (warp == 6) {
    // ---------------- slab manager: residual loads and output stores ----------------
    // Slab sn (four per tile, 32 channels each) lives in buffer sn % kSlabs; its store is
    // issued once the 128 epilogue threads have written it, and once that store has read
    // the buffer the residual of slab sn + kSlabs is loaded into it.
    if (lane == 0) {
      bool ok = true;
      const int total = 4 * n_mine;
      auto coords = [&](int sn, int& cc, int& j0, int& r, int& b) {
        const int tile = blockIdx.x + (sn >> 2) * gridDim.x;
        const int jt = tile % n_jt, rb = tile / n_jt;
        cc = sn & 3;
        j0 = jt * 128;
        r = rb % rows;
        b = rb / rows;
      };
      auto load = [&](int sn) {
        const int sl = sn % kSlabs;
        if (add_residual) {
          int cc, j0, r, b;
          coords(sn, cc, j0, r, b);
          mbar_arrive_expect_tx(&bars->o_full[sl], 16384);
          tma_load_4d(smem + kO + sl * 16384, &z_map, &bars->o_full[sl], cc * 32, j0, r, b);
        } else {
          mbar_arrive(&bars->o_full[sl]);
        }
      };
      int loaded = 0;
      for (; loaded < kSlabs && loaded < total; ++loaded) load(loaded);
      for (int sn = 0; sn < total; ++sn) {
        const int sl = sn % kSlabs;
        if (!mbar_wait(&bars->slab_ready[sl], (sn / kSlabs) & 1, guard, status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        int cc, j0, r, b;
        coords(sn, cc, j0, r, b);
        tma_store_4d(&out_map, smem + kO + sl * 16384, cc * 32, j0, r, b);
        tma_store_commit();
        if (sn + kSlabs < total) {
          tma_store_wait_read();  // the store has read the buffer
          load(sn + kSlabs);
          ++loaded;
        }
      }
      tma_store_wait_all();
      if (!ok)  // let the residual loads still in flight land before shared memory is released
        for (int t = (loaded > kSlabs ? loaded - kSlabs : 0); t < loaded; ++t)
          mbar_wait_drain(&bars->o_full[t % kSlabs], (t / kSlabs) & 1);
    }
  } else if (warp < 4) {
    // ------------------------- epilogue: thread = pair -------------------------
    const int p = tid;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    int slab = 0;
    bool ok = true;
    for (int it = 0; ok && it < n_mine; ++it) {
      const int s = it & 1;
      const int tile = blockIdx.x + it * gridDim.x;
      const int jt = tile % n_jt, rb = tile / n_jt;
      const int j = jt * 128 + p;
      // the pair's mask value (1 without a mask), loaded before the wait hides its latency
      const float mv = (mask && j < N) ? __ldg(mask + static_cast<size_t>(rb) * N + j) : 1.f;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[s], (it >> 1) & 1, guard, status, kStatusTimeoutConsumer));
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc, ++slab) {
        const int sl = slab % kSlabs;
        uint32_t d[32];
        tmem_ld32(tmem + lane_off + s * 128 + cc * 32, d);
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_full[sl], (slab / kSlabs) & 1, guard, status,
                                               kStatusTimeoutConsumer));
        tmem_wait_ld();
        if (!ok) break;
        uint8_t* ob = smem + kO + sl * 16384;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int n = cc * 32 + q * 4;
          const float4 bb = *reinterpret_cast<const float4*>(sb2 + n);
          float4 o = make_float4(__uint_as_float(d[q * 4 + 0]) + bb.x, __uint_as_float(d[q * 4 + 1]) + bb.y,
                                 __uint_as_float(d[q * 4 + 2]) + bb.z, __uint_as_float(d[q * 4 + 3]) + bb.w);
          if (add_residual) {
            const float4 zv = lds_f4(ob + swz128(p, q));
            o.x += zv.x;
            o.y += zv.y;
            o.z += zv.z;
            o.w += zv.w;
          }
          o.x *= mv;
          o.y *= mv;
          o.z *= mv;
          o.w *= mv;
          *reinterpret_cast<float4*>(ob + swz128(p, q)) = o;
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->slab_ready[sl]);  // warp 6 stores the slab
      }
      if (!ok) break;
      tc_fence_before();
      mbar_arrive(&bars->d_empty[s]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ----------------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------------
// hidden rows [B*N*N][512] fp16 addressed as (unit, j, b*N + i); box (64, 128, 1), 128-B swizzle
static int make_hid_map(CUtensorMap* m, const void* base, int64_t BR, int64_t N) {
  uint64_t dims[3] = {static_cast<uint64_t>(tnpack::kHid), static_cast<uint64_t>(N), static_cast<uint64_t>(BR)};
  uint64_t strides[2] = {tnpack::kHid * 2, static_cast<uint64_t>(N) * tnpack::kHid * 2};
  uint32_t box[3] = {64, 128, 1};
  return encode_tmap(m, TmaType::kF16, 3, base, dims, strides, box, 128);
}

// W2 [128][512] fp16 addressed as (k, out); box (64 k, 128 rows), 128-B swizzle
static int make_w2_map(CUtensorMap* m, const void* base) {
  uint64_t dims[2] = {static_cast<uint64_t>(tnpack::kHid), static_cast<uint64_t>(tnpack::kCp)};
  uint64_t strides[1] = {tnpack::kHid * 2};
  uint32_t box[2] = {64, 128};
  return encode_tmap(m, TmaType::kF16, 2, base, dims, strides, box, 128);
}

static int transition_check(int c_p, int n) {
  if (c_p != tnpack::kCp || n < 1 || n > tnpack::kHid / tnpack::kCp)
    return fail(GTK_ERR_UNSUPPORTED, "transition: the tuned kernels take c_p = 128 with n <= 4");
  return GTK_OK;
}

}  // namespace gtk

using namespace gtk;

extern "C" {

// The tuned kernels: c_p = 128 with n <= 4 (n < 4 zero-padded to 512 hidden units when packed).
static bool transition_tuned(int c_p, int n) { return c_p == tnpack::kCp && n >= 1 && n <= tnpack::kHid / tnpack::kCp; }

size_t gtk_transition_packed_bytes(int c_p, int n) {
  return transition_tuned(c_p, n) ? tnpack::kBytes : gen::transition_packed_bytes(c_p, n);
}

size_t gtk_transition_workspace_bytes(int64_t B, int64_t N, int c_p, int n) {
  if (!transition_tuned(c_p, n)) return gen::transition_workspace_bytes(B, N, c_p, n);
  if (B < 1 || N < 1) return 0;
  return static_cast<size_t>(B) * N * N * tnpack::kHid * 2;
}

int gtk_transition_pack(const gtk_transition_params* params, int c_p, int n, void* packed, size_t packed_bytes,
                        void* stream) {
  if (!transition_tuned(c_p, n)) return gen::transition_pack(params, c_p, n, packed, packed_bytes, stream);
  if (int e = transition_check(c_p, n)) return e;
  if (!params || !params->ln_w || !params->ln_b || !params->w1 || !params->w2)
    return fail(GTK_ERR_INVALID_ARG, "transition_pack: a required parameter pointer is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < tnpack::kBytes) return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  if (int e = check_device()) return e;
  transition_pack_kernel<<<64, 256, 0, static_cast<cudaStream_t>(stream)>>>(*params, static_cast<uint8_t*>(packed),
                                                                            n * tnpack::kCp);
  return check_launch("transition_pack_kernel");
}

int gtk_transition_forward(const float* z, const float* mask, const void* packed, float* out, int add_residual,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_p, int n,
                           uint32_t* status, void* stream) {
  if (!transition_tuned(c_p, n))  // every other shape: the general path
    return gen::transition_forward(z, mask, packed, out, add_residual, workspace, workspace_bytes, B, N, c_p, n, status,
                                   stream);
  if (int e = transition_check(c_p, n)) return e;
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535)) return fail(GTK_ERR_INVALID_ARG, "transition: bad B/N");
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(out, "out")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (workspace_bytes < gtk_transition_workspace_bytes(B, N, c_p, n))
    return fail(GTK_ERR_WORKSPACE, "transition: workspace too small");
  if (int e = check_device()) return e;
  const int64_t n_jt = (N + 127) / 128;
  const int64_t n_tiles = B * N * n_jt;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "transition: too many tiles");
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  const float* vec = reinterpret_cast<const float*>(pk + tnpack::kVec);
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    CUtensorMap wm, zm;
    if (int e = make_weight_map(&wm, pk + tnpack::kW1, tnpack::kHid, 128)) return e;
    if (int e = make_pair_map(&zm, z, B, N, N, false)) return e;
    if (int e = ensure_smem(reinterpret_cast<const void*>(transition_in_kernel), k5a::kSmem)) return e;
    transition_in_kernel<<<grid, k5a::kThreads, k5a::kSmem, st>>>(wm, zm, vec, static_cast<__half*>(workspace),
                                                                   static_cast<int>(N), static_cast<int>(N),
                                                                   static_cast<int>(n_jt), static_cast<int>(n_tiles),
                                                                   status);
    if (int e = check_launch("transition_in_kernel")) return e;
  }
  CUtensorMap hm, wm, zm, om;
  if (int e = make_hid_map(&hm, workspace, B * N, N)) return e;
  if (int e = make_w2_map(&wm, pk + tnpack::kW2)) return e;
  if (int e = make_pair_map(&zm, add_residual ? z : out, B, N, N, false)) return e;
  if (int e = make_pair_map(&om, out, B, N, N, false)) return e;
  if (int e = ensure_smem(reinterpret_cast<const void*>(transition_out_kernel), k5b::kSmem)) return e;
  transition_out_kernel<<<grid, k5b::kThreads, k5b::kSmem, st>>>(hm, wm, zm, om, vec, mask, static_cast<int>(N),
                                                                  static_cast<int>(N), add_residual,
                                                                  static_cast<int>(n_jt), static_cast<int>(n_tiles),
                                                                  status);
  return check_launch("transition_out_kernel");
}

}  // extern "C"
