// Pair embedding producer (reference examples/basic_usage.py:181-199): the initial pair
// representation p[b,i,j] = Linear(2 c_s -> c_p)([s_i ; s_j]) and the pair mask
// p_mask[b,i,j] = mask[b,i] * mask[b,j], written straight into the fp32 pair layout
// [B, rows, N, c_p] (a row shard when rows < N), so the concatenated [B, N, N, 2 c_s] tensor
// of the reference is never formed.
//
// With W = [W_a | W_b] split along the input, p[b,i,j] = U[b,i] + V[b,j] where
// U = s W_a^T and V = s W_b^T + bias. Two kernels:
//   E1 embed_project_kernel  U and V (fp32, [B*N][c_p] each): a 64 x 128 x c_s tiled fp32
//                            GEMM on the CUDA cores (2 B N c_s c_p MACs -- about 0.1 GFLOP
//                            at N = 1024, c_s = 384 -- in fp32 like the reference's Linear);
//   E2 embed_pairs_kernel    the broadcast sum, one warp per pair row segment: HBM write
//                            bound at 512 B per pair (+ 4 B for the mask).
#include <cuda_runtime.h>

#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {

namespace embed {
constexpr int kCp = 128;
constexpr int kRows = 64;   // rows of s per E1 block
constexpr int kKc = 32;     // K chunk
constexpr int kThreads1 = 256;
}  // namespace embed

// E1: out[which][r][n] = sum_k s[r][k] * w[n][which * c_s + k] (+ bias[n] for which = 1).
// Block: 64 rows x 128 outputs of one `which`; thread (ty, tx) in 16 x 16 owns rows
// ty*4..+3 and outputs tx + 16*q (q = 0..7): a 4 x 8 register tile.
__global__ void __launch_bounds__(embed::kThreads1)
    embed_project_kernel(const float* __restrict__ s, const float* __restrict__ w, const float* __restrict__ bias,
                         float* __restrict__ uv, int64_t BN, int c_s) {
  using namespace embed;
  __shared__ float s_t[kKc][kRows + 1];  // [k][row]
  __shared__ float w_t[kKc][kCp + 1];    // [k][out]
  const int which = blockIdx.y;          // 0: U (W_a), 1: V (W_b)
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRows;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[a][q] = 0.f;
  const int64_t ldw = 2 * static_cast<int64_t>(c_s);
  for (int k0 = 0; k0 < c_s; k0 += kKc) {
    // stage s[r0 .. r0+63][k0 .. k0+31] and w[0..127][which*c_s + k0 .. +31], transposed
    for (int e = threadIdx.x; e < kRows * kKc; e += kThreads1) {
      const int r = e / kKc, k = e % kKc;
      const int64_t gr = r0 + r;
      s_t[k][r] = (gr < BN && k0 + k < c_s) ? s[gr * c_s + k0 + k] : 0.f;
    }
    for (int e = threadIdx.x; e < kCp * kKc; e += kThreads1) {
      const int n = e / kKc, k = e % kKc;
      w_t[k][n] = (k0 + k < c_s) ? w[n * ldw + which * c_s + k0 + k] : 0.f;
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
  float* out = uv + static_cast<int64_t>(which) * BN * kCp;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t gr = r0 + ty * 4 + a;
    if (gr >= BN) continue;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int n = tx + 16 * q;
      out[gr * kCp + n] = acc[a][q] + ((which == 1 && bias) ? bias[n] : 0.f);
    }
  }
}

// E2: out[b, r, j, :] = U[b, row0 + r, :] + V[b, j, :]; pair_mask[b, r, j] = m[b, row0 + r] m[b, j].
// One warp per (b, r, 32-pair segment of j): lane l owns channels 4l .. 4l+3, so each pair
// row (512 B) is one 16-byte load of V (L2-resident: V is 512 B per residue) and one
// 16-byte streaming store per lane, every warp store covering the pair's 512 contiguous
// bytes. The grid-stride loop runs over (b, r, segment).
__global__ void __launch_bounds__(256)
    embed_pairs_kernel(const float* __restrict__ uv, const float* __restrict__ mask, float* __restrict__ out,
                       float* __restrict__ pair_mask, int64_t B, int64_t N, int64_t rows, int64_t row0) {
  using namespace embed;
  const float4* U = reinterpret_cast<const float4*>(uv);
  const float4* V = reinterpret_cast<const float4*>(uv + B * N * kCp);
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t nseg = (N + 31) / 32;
  const int64_t total = B * rows * nseg;
  for (int64_t t = warp; t < total; t += nwarps) {
    const int64_t seg = t % nseg, br = t / nseg;
    const int64_t r = br % rows, b = br / rows;
    const int64_t i = row0 + r;
    const float4 u = __ldg(U + (b * N + i) * (kCp / 4) + lane);
    const int64_t j0 = seg * 32;
    const int jn = static_cast<int>((N - j0) < 32 ? (N - j0) : 32);
    float4* orow = reinterpret_cast<float4*>(out + ((b * rows + r) * N + j0) * kCp);
    const float4* vseg = V + (b * N + j0) * (kCp / 4) + lane;
#pragma unroll 4
    for (int jj = 0; jj < jn; ++jj) {
      const float4 v = __ldg(vseg + jj * (kCp / 4));
      __stcs(orow + jj * (kCp / 4) + lane, make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w));
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
  if (c_p != embed::kCp || B < 1 || N < 1) return 0;
  return static_cast<size_t>(2) * B * N * embed::kCp * sizeof(float);
}

int gtk_pair_embed(const float* s, const float* mask, const float* weight, const float* bias, float* out,
                   float* pair_mask, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int64_t rows,
                   int64_t row0, int c_s, int c_p, void* stream) {
  if (c_p != embed::kCp) return fail(GTK_ERR_UNSUPPORTED, "pair_embed: c_p must be 128");
  if (c_s < 1 || c_s > 65536) return fail(GTK_ERR_INVALID_ARG, "pair_embed: bad c_s");
  if (!dims_ok(B, 65535) || !dims_ok(N, 1 << 20) || !dims_ok(rows, N) || row0 < 0 || row0 + rows > N)
    return fail(GTK_ERR_INVALID_ARG, "pair_embed: bad B/N/rows/row0");
  if (int e = check_ptr(s, "s", 4)) return e;
  if (int e = check_ptr(weight, "weight", 4)) return e;
  if (int e = check_ptr(out, "out")) return e;
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
  dim3 g1(static_cast<unsigned>((BN + embed::kRows - 1) / embed::kRows), 2);
  embed_project_kernel<<<g1, embed::kThreads1, 0, st>>>(s, weight, bias, uv, BN, c_s);
  if (int e = check_launch("embed_project_kernel")) return e;
  const int64_t warps = B * rows * ((N + 31) / 32);
  const int64_t blocks_needed = (warps + 7) / 8;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  const int blocks = static_cast<int>(blocks_needed < cap ? blocks_needed : cap);
  embed_pairs_kernel<<<blocks, 256, 0, st>>>(uv, mask, out, pair_mask, B, N, rows, row0);
  return check_launch("embed_pairs_kernel");
}

}  // extern "C"
