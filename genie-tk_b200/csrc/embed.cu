// Pair embedding producer (reference examples/basic_usage.py:181-199): the initial pair
// representation p[b,i,j] = Linear(2 c_s -> c_p)([s_i ; s_j]) and the pair mask
// p_mask[b,i,j] = mask[b,i] * mask[b,j], written straight into the fp32 pair layout
// [B, rows, N, c_p] (a row shard when rows < N), so the concatenated [B, N, N, 2 c_s] tensor
// of the reference is never formed.
//
// With W = [W_a | W_b] split along the input, p[b,i,j] = U[b,i] + V[b,j] where
// U = s W_a^T and V = s W_b^T + bias. Two kernels:
//   E1 embed_project_kernel  U and V (fp32, [B*N][c_p] each): a 64 x 128 x c_s tiled fp32
//                            GEMM on the CUDA cores, one block per 64 rows and 128-output
//                            chunk (2 B N c_s c_p MACs -- about 0.1 GFLOP at N = 1024,
//                            c_s = 384, c_p = 128 -- in fp32 like the reference's Linear);
//   E2 embed_pairs_kernel    the broadcast sum, one warp per pair row segment: HBM write
//                            bound at 4 c_p B per pair (+ 4 B for the mask).
// Any c_p in 1..4096; 16-byte vectors when c_p is a multiple of 4, single floats otherwise.
#include <cuda_runtime.h>

#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {

namespace embed {
constexpr int kCp = 128;    // outputs per E1 block
constexpr int kMaxCp = 4096;
constexpr int kRows = 64;   // rows of s per E1 block
constexpr int kKc = 32;     // K chunk
constexpr int kThreads1 = 256;
}  // namespace embed

// E1: out[which][r][n] = sum_k s[r][k] * w[n][which * c_s + k] (+ bias[n] for which = 1).
// Block (x, y): rows 64x .. 64x+63, output chunk n0 = 128 (y / 2) of which = y % 2. Thread
// (ty, tx) in 16 x 16 owns rows ty*4..+3 and outputs n0 + tx + 16*q (q = 0..7): a 4 x 8
// register tile.
__global__ void __launch_bounds__(embed::kThreads1)
    embed_project_kernel(const float* __restrict__ s, const float* __restrict__ w, const float* __restrict__ bias,
                         float* __restrict__ uv, int64_t BN, int c_s, int c_p) {
  using namespace embed;
  __shared__ float s_t[kKc][kRows + 1];  // [k][row]
  __shared__ float w_t[kKc][kCp + 1];    // [k][out]
  const int which = blockIdx.y & 1;      // 0: U (W_a), 1: V (W_b)
  const int n0 = (blockIdx.y >> 1) * kCp;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[a][q] = 0.f;
  const int64_t ldw = 2 * static_cast<int64_t>(c_s);
  for (int k0 = 0; k0 < c_s; k0 += kKc) {
    // stage s[r0 .. r0+63][k0 .. k0+31] and w[n0 .. n0+127][which*c_s + k0 .. +31], transposed
    for (int e = threadIdx.x; e < kRows * kKc; e += kThreads1) {
      const int r = e / kKc, k = e % kKc;
      const int64_t gr = r0 + r;
      s_t[k][r] = (gr < BN && k0 + k < c_s) ? s[gr * c_s + k0 + k] : 0.f;
    }
    for (int e = threadIdx.x; e < kCp * kKc; e += kThreads1) {
      const int n = e / kKc, k = e % kKc;
      w_t[k][n] = (n0 + n < c_p && k0 + k < c_s) ? w[(n0 + n) * ldw + which * c_s + k0 + k] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kKc; ++k) {
      float sv[4], wv[8];
#pragma unroll
      for (int a = 0; a < 4; ++a) sv[a] = s_t[k][ty * 4 + a];
#pragma unroll
      for (int q = 0; q < 8; ++q) wv[q] = w_t[k][tx + 16 * q];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[a][q] = fmaf(sv[a], wv[q], acc[a][q]);
    }
    __syncthreads();
  }
  float* out = uv + static_cast<int64_t>(which) * BN * c_p;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t gr = r0 + ty * 4 + a;
    if (gr >= BN) continue;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int n = n0 + tx + 16 * q;
      if (n < c_p) out[gr * c_p + n] = acc[a][q] + ((which == 1 && bias) ? bias[n] : 0.f);
    }
  }
}

// E2: out[b, r, j, :] = U[b, row0 + r, :] + V[b, j, :]; pair_mask[b, r, j] = m[b, row0 + r] m[b, j].
// One warp per (b, r, 32-pair segment of j). With kVec (c_p a multiple of 4) the lanes walk
// each pair row in 16-byte vectors, so every warp store covers 512 contiguous bytes of it (at
// c_p = 128 lane l owns channels 4l .. 4l+3 and keeps its slice of U in registers; V is
// L2-resident, 4 c_p B per residue); otherwise single floats. The grid-stride loop runs over
// (b, r, segment).
template <bool kVec>
__global__ void __launch_bounds__(256)
    embed_pairs_kernel(const float* __restrict__ uv, const float* __restrict__ mask, float* __restrict__ out,
                       float* __restrict__ pair_mask, int64_t B, int64_t N, int64_t rows, int64_t row0, int c_p) {
  const float* U = uv;
  const float* V = uv + B * N * c_p;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t nseg = (N + 31) / 32;
  const int64_t total = B * rows * nseg;
  const int nv = kVec ? c_p / 4 : c_p;  // vectors per pair row
  for (int64_t t = warp; t < total; t += nwarps) {
    const int64_t seg = t % nseg, br = t / nseg;
    const int64_t r = br % rows, b = br / rows;
    const int64_t i = row0 + r;
    const int64_t j0 = seg * 32;
    const int jn = static_cast<int>((N - j0) < 32 ? (N - j0) : 32);
    float* orow = out + ((b * rows + r) * N + j0) * c_p;
    const float* urow = U + (b * N + i) * c_p;
    const float* vseg = V + (b * N + j0) * c_p;
    if (kVec) {
      const float4* u4 = reinterpret_cast<const float4*>(urow);
      if (nv == 32) {
        const float4 u = __ldg(u4 + lane);
#pragma unroll 4
        for (int jj = 0; jj < jn; ++jj) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(vseg + jj * c_p) + lane);
          __stcs(reinterpret_cast<float4*>(orow + jj * c_p) + lane, make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w));
        }
      } else {
        for (int jj = 0; jj < jn; ++jj)
          for (int e = lane; e < nv; e += 32) {
            const float4 u = __ldg(u4 + e);
            const float4 v = __ldg(reinterpret_cast<const float4*>(vseg + jj * c_p) + e);
            __stcs(reinterpret_cast<float4*>(orow + jj * c_p) + e, make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w));
          }
      }
    } else {
      for (int jj = 0; jj < jn; ++jj)
        for (int e = lane; e < nv; e += 32) __stcs(orow + jj * c_p + e, __ldg(urow + e) + __ldg(vseg + jj * c_p + e));
    }
    if (pair_mask && lane < jn) {
      const float mi = mask ? __ldg(mask + b * N + i) : 1.f;
      pair_mask[(b * rows + r) * N + j0 + lane] = mi * (mask ? __ldg(mask + b * N + j0 + lane) : 1.f);
    }
  }
}

}  // namespace gtk

using namespace gtk;

extern "C" {

size_t gtk_pair_embed_workspace_bytes(int64_t B, int64_t N, int c_p) {
  if (c_p < 1 || c_p > embed::kMaxCp || B < 1 || N < 1) return 0;
  return static_cast<size_t>(2) * B * N * c_p * sizeof(float);
}

int gtk_pair_embed(const float* s, const float* mask, const float* weight, const float* bias, float* out,
                   float* pair_mask, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int64_t rows,
                   int64_t row0, int c_s, int c_p, void* stream) {
  if (c_p < 1 || c_p > embed::kMaxCp)
    return fail(GTK_ERR_UNSUPPORTED, "pair_embed: c_p must lie in 1.." + std::to_string(embed::kMaxCp));
  if (c_s < 1 || c_s > 65536) return fail(GTK_ERR_INVALID_ARG, "pair_embed: bad c_s");
  if (!dims_ok(B, 65535) || !dims_ok(N, 1 << 20) || !dims_ok(rows, N) || row0 < 0 || row0 + rows > N)
    return fail(GTK_ERR_INVALID_ARG, "pair_embed: bad B/N/rows/row0");
  if (int e = check_ptr(s, "s", 4)) return e;
  if (int e = check_ptr(weight, "weight", 4)) return e;
  // 16-byte vectors need a 16-byte aligned output (and workspace) and whole vectors per row
  const bool vec = (c_p % 4) == 0;
  if (int e = check_ptr(out, "out", vec ? 16 : 4)) return e;
  if (int e = check_ptr(workspace, "workspace")) return e;
  if (bias && (reinterpret_cast<uintptr_t>(bias) & 3)) return fail(GTK_ERR_ALIGNMENT, "bias is misaligned");
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (pair_mask && (reinterpret_cast<uintptr_t>(pair_mask) & 3))
    return fail(GTK_ERR_ALIGNMENT, "pair_mask is misaligned");
  if (workspace_bytes < gtk_pair_embed_workspace_bytes(B, N, c_p))
    return fail(GTK_ERR_WORKSPACE, "pair_embed: workspace too small");
  if (int e = check_device()) return e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t BN = B * N;
  float* uv = static_cast<float*>(workspace);
  const int chunks = (c_p + embed::kCp - 1) / embed::kCp;
  dim3 g1(static_cast<unsigned>((BN + embed::kRows - 1) / embed::kRows), static_cast<unsigned>(2 * chunks));
  embed_project_kernel<<<g1, embed::kThreads1, 0, st>>>(s, weight, bias, uv, BN, c_s, c_p);
  if (int e = check_launch("embed_project_kernel")) return e;
  const int64_t warps = B * rows * ((N + 31) / 32);
  const int64_t blocks_needed = (warps + 7) / 8;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  const int blocks = static_cast<int>(blocks_needed < cap ? blocks_needed : cap);
  if (vec)
    embed_pairs_kernel<true><<<blocks, 256, 0, st>>>(uv, mask, out, pair_mask, B, N, rows, row0, c_p);
  else
    embed_pairs_kernel<false><<<blocks, 256, 0, st>>>(uv, mask, out, pair_mask, B, N, rows, row0, c_p);
  return check_launch("embed_pairs_kernel");
}

}  // extern "C"
