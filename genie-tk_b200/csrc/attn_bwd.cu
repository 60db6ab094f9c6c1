// The triangle-attention core for training -- forward with the softmax statistics and its
// backward, without ever forming the [B, N, H, N, N] score tensor -- and the generic gated
// multi-head attention core of the reference's Attention module.
//
// Frame of the block (z itself for the starting node, z^T for the ending node), pair row i,
// query j, key k, head h, head_dim d (reference primitives.py:134-164):
//   s[i,h,j,k] = q[i,j,h] . k[i,k,h] / sqrt(d) + inf * (m[i,k] - 1) + tri[h,j,k]
//   p = softmax_k(s),  o[i,j,h] = sum_k p v[i,k,h]
// With D = sum_e do o per (i, j, h) and ds = p (do . v_k - D):
//   dq[i,j] = sum_k ds k[i,k] / sqrt(d)          (query-major kernel)
//   dk[i,k] = sum_j ds q[i,j] / sqrt(d),  dv[i,k] = sum_j p do[i,j]   (key-major kernel)
//   dtri[h,j,k] = sum_i ds[i,h,j,k]              (bias-major: CTA = query block x key block)
//
// Operands. q, k, v and do enter as fp16 planes [B, N(i), H, N(j), Dp] (Dp = head_dim rounded
// up to 16, 32 or 64, zero-padded; do times a power-of-two scale), the triangle bias as fp16
// [B, H, N(j), Np] (Np = N rounded up to 8), written by gtk_attn_core_pack /
// gtk_attn_core_pack_bias from the fp32 projections: every 64-row tile of a plane is one
// contiguous block, which cp.async copies 16 bytes at a time into shared memory, double
// buffered so that the next tile lands while the tensor cores work on this one. The mask
// stays fp32 [B, N(i), N(k)] (or NULL), outputs and gradients are fp32 in the projections'
// layout [B, N(i), N(j), H*d] and [B, H, N(j), N(k)]. The statistics are, per (b, i, h, j),
// the running max m of the base-2 scores and 1 / l, l = sum_k 2^(s2 - m), kept apart: for a
// fully masked row every score is about -1.4e9, and m + log2 l would round back to m.
//
// Arithmetic: every product runs on the tensor cores as mma.sync m16n8k16 (fp16 operands,
// fp32 accumulation); the scores get their scale, bias and mask in fp32, softmax and ds are
// fp32. A CTA is four warps; a warp owns 16 of the CTA's 64 rows and keeps its operand
// fragments in registers, and the score / probability fragments are reused in place as the A
// operand of the next product.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "attn_core.h"
#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kRows = 64;      // rows (queries or keys) per CTA and per staged tile
constexpr int kThreads = 128;  // four warps of 16 rows
constexpr int kBP = kRows + 8; // pitch (halves) of a staged 64 x 64 bias tile

struct Args {
  const __half* q;     // [B][N][H][N][Dp]
  const __half* k;
  const __half* v;
  const __half* tri;   // [B][H][N][Np]
  const float* mask;   // [B] planes of N x N, element (i, k) at i * msi + k * msk; or NULL
  const float2* stat;  // (m, 1 / l) per [b][i][h][j]
  const __half* dO;    // [B][N][H][N][Dp], times gscale
  const float* dsum;   // D[b][i][h][j] (unscaled)
  float* out_o;
  float2* out_stat;
  float* dq;
  float* dk;
  float* dv;
  float* dtri;
  int64_t N, Np;
  int64_t msi, msk;  // mask strides: (N, 1) in the block's frame, (1, N) for z^T's frame
  int H, d, hd;
  float qscale;   // log2 e / sqrt(d)
  float inf2;     // inf * log2 e
  float gscale;   // power-of-two scale of dO in its fp16 plane
};

// ------------------------------- warp-level tensor-core helpers --------------------------
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const __half* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const __half* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

__device__ __forceinline__ uint32_t h2(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 16-byte global -> shared copy; zero-fills the 16 bytes when `valid` is false (the source
// address is then never read, but is kept inside the plane).
__device__ __forceinline__ void cp16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kPending) : "memory");
}

// Rows r0 .. r0+63 of a packed plane (row pitch D halves, `N` rows) into a staged tile of
// pitch D + 8; rows past N are zero.
template <int D>
__device__ __forceinline__ void load_rows(__half (*t)[D + 8], const __half* __restrict__ src, int64_t r0, int64_t N) {
  constexpr int C = D / 8;
  for (int idx = threadIdx.x; idx < kRows * C; idx += kThreads) {
    const int r = idx / C, c = idx - r * C;
    const bool ok = r0 + r < N;
    cp16(&t[r][c * 8], src + (ok ? r0 + r : 0) * D + c * 8, ok);
  }
}

// The 64 x 64 block (rows r0.., columns c0..) of a packed bias plane (row pitch Np).
__device__ __forceinline__ void load_bias(__half (*t)[kBP], const __half* __restrict__ src, int64_t r0, int64_t c0,
                                          int64_t N, int64_t Np) {
  for (int idx = threadIdx.x; idx < kRows * 8; idx += kThreads) {
    const int r = idx >> 3, c = idx & 7;
    const bool ok = r0 + r < N && c0 + c * 8 < Np;
    cp16(&t[r][c * 8], src + (ok ? (r0 + r) * Np + c0 + c * 8 : 0), ok);
  }
}

// A fragments (16 rows x 16 columns, row-major) of the warp's rows for every 16-column step.
template <int D>
__device__ __forceinline__ void load_a(uint32_t (&f)[D / 16][4], const __half (*t)[D + 8], int row0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) ldsm_x4(f[kk], &t[row0 + (lane & 15)][kk * 16 + (lane >> 4) * 8]);
}

// c[0..1] += A (16 x D) . T[n0 .. n0+15]^T: the tile's rows are the product's columns
// (S = Q K^T with K's rows as keys).
template <int D>
__device__ __forceinline__ void mma_abt(float (&c)[2][4], const uint32_t (&a)[D / 16][4], const __half (*t)[D + 8],
                                        int n0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t b[4];
    ldsm_x4(b, &t[n0 + (lane & 7) + ((lane >> 4) << 3)][kk * 16 + ((lane >> 3) & 1) * 8]);
    mma16816(c[0], a[kk], b[0], b[1]);
    mma16816(c[1], a[kk], b[2], b[3]);
  }
}

// acc (16 x D) += A (16 x 16) . T[k0 .. k0+15][0 .. D): the tile's rows are the reduction
// (O += P V with V's rows as keys).
template <int D>
__device__ __forceinline__ void mma_at(float (&acc)[D / 8][4], const uint32_t (&a)[4], const __half (*t)[D + 8],
                                       int k0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int dn = 0; dn < D / 16; ++dn) {
    uint32_t b[4];
    ldsm_x4_t(b, &t[k0 + (lane & 7) + ((lane >> 3) & 1) * 8][dn * 16 + (lane >> 4) * 8]);
    mma16816(acc[2 * dn], a, b[0], b[1]);
    mma16816(acc[2 * dn + 1], a, b[2], b[3]);
  }
}

// Two 16 x 8 accumulators (columns c0 .. c0+15) as the A operand of the next product.
__device__ __forceinline__ void c_to_a(uint32_t (&a)[4], const float (&c)[2][4]) {
  a[0] = h2(c[0][0], c[0][1]);
  a[1] = h2(c[0][2], c[0][3]);
  a[2] = h2(c[1][0], c[1][1]);
  a[3] = h2(c[1][2], c[1][3]);
}

// Accumulator element i of a 16 x 8 block: row (lane >> 2) + 8 (i >> 1), column 2 (lane & 3) + (i & 1).
__device__ __forceinline__ int c_row(int i) { return ((threadIdx.x & 31) >> 2) + ((i >> 1) << 3); }
__device__ __forceinline__ int c_col(int i) { return 2 * (threadIdx.x & 3) + (i & 1); }

// The mask row of pair row `row` = b * N + i (NULL without a mask).
__device__ __forceinline__ const float* mask_row(const Args& a, int64_t row) {
  if (!a.mask) return nullptr;
  const int64_t b = row / a.N, i = row - b * a.N;
  return a.mask + b * a.N * a.N + i * a.msi;
}

// inf * (m - 1) in base-2 units for key k of a mask row; -inf past the last key.
__device__ __forceinline__ float mask_bias2(const Args& a, const float* mrow, int64_t k) {
  if (k >= a.N) return -INFINITY;
  return mrow ? a.inf2 * (mrow[k * a.msk] - 1.f) : 0.f;
}

__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}

__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  return x + __shfl_xor_sync(0xffffffffu, x, 2);
}

__device__ __forceinline__ float2 bias_pair(const __half (*b)[kBP], int r, int c) {
  return __half22float2(*reinterpret_cast<const __half2*>(&b[r][c]));
}

// Shared memory of the query-major kernels (forward and dq): two stages of a key tile, a
// value tile (or the output-gradient tile's partner), the bias block and the mask bias.
template <int D>
struct RowSmem {
  __half k[2][kRows][D + 8];
  __half v[2][kRows][D + 8];
  __half b[2][kRows][kBP];
  float m[2][kRows];
};

// Shared memory of the key-major kernel: two stages of the query and output-gradient tiles,
// the bias block and the statistics of the tile's queries.
template <int D>
struct ColSmem {
  __half q[2][kRows][D + 8];
  __half g[2][kRows][D + 8];
  __half b[2][kRows][kBP];
  float2 l[2][kRows];
  float dsum[2][kRows];
};

// Shared memory of the bias-gradient kernel: two stages of one pair row's q, do, k, v tiles.
template <int D>
struct TriSmem {
  __half q[2][kRows][D + 8];
  __half g[2][kRows][D + 8];
  __half k[2][kRows][D + 8];
  __half v[2][kRows][D + 8];
  __half bias[kRows][kBP];  // the CTA's 64 x 64 bias block, loaded once
  float m[2][kRows];
  float2 l[2][kRows];
  float dsum[2][kRows];
};

// Base of the (pair row, head) slice of a packed plane.
template <int D>
__device__ __forceinline__ const __half* plane(const __half* p, const Args& a, int64_t row, int h) {
  return p + (row * a.H + h) * a.N * D;
}

// ---------------------------------------------------------------------------------------
// Forward with statistics. CTA = (pair row b*N+i, head h, 64 queries); warp = 16 queries.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) fwd_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RowSmem<D>& S = *reinterpret_cast<RowSmem<D>*>(smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int h = blockIdx.y;
  const int64_t row = blockIdx.x, N = a.N, b = row / N;
  const int64_t j0 = static_cast<int64_t>(blockIdx.z) * kRows;
  const __half* qp = plane<D>(a.q, a, row, h);
  const __half* kp = plane<D>(a.k, a, row, h);
  const __half* vp = plane<D>(a.v, a, row, h);
  const __half* bp = a.tri + (b * a.H + h) * N * a.Np;
  const float* mrow = mask_row(a, row);
  const int nt = static_cast<int>((N + kRows - 1) / kRows);
  auto issue = [&](int t, int st) {
    const int64_t k0 = static_cast<int64_t>(t) * kRows;
    load_rows<D>(S.k[st], kp, k0, N);
    load_rows<D>(S.v[st], vp, k0, N);
    load_bias(S.b[st], bp, j0, k0, N, a.Np);
    if (threadIdx.x < kRows) S.m[st][threadIdx.x] = mask_bias2(a, mrow, k0 + threadIdx.x);
  };
  load_rows<D>(S.k[1], qp, j0, N);  // q passes through stage 1's key buffer
  issue(0, 0);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  uint32_t qf[D / 16][4];
  load_a<D>(qf, S.k[1], w * 16);
  __syncthreads();
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int jl0 = w * 16 + (lane >> 2);
  for (int t = 0; t < nt; ++t) {
    const int st = t & 1;
    if (t + 1 < nt) issue(t + 1, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    float s[4][2][4];
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int x = 0; x < 2; ++x) s[np][x][0] = s[np][x][1] = s[np][x][2] = s[np][x][3] = 0.f;
      mma_abt<D>(s[np], qf, S.k[st], np * 16);
    }
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int np = 0; np < 4; ++np)
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int kl = np * 16 + x * 8 + 2 * (lane & 3);
          const float2 bb = bias_pair(S.b[st], jl0 + 8 * r, kl);
          const float v0 = fmaf(s[np][x][2 * r], a.qscale, fmaf(bb.x, kLog2e, S.m[st][kl]));
          const float v1 = fmaf(s[np][x][2 * r + 1], a.qscale, fmaf(bb.y, kLog2e, S.m[st][kl + 1]));
          s[np][x][2 * r] = v0;
          s[np][x][2 * r + 1] = v1;
          tmax[r] = fmaxf(tmax[r], fmaxf(v0, v1));
        }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mnew = fmaxf(m[r], quad_max(tmax[r]));
      const float corr = exp2f(m[r] - mnew);  // 0 on the first tile (m = -inf)
      l[r] *= corr;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        o[n][2 * r] *= corr;
        o[n][2 * r + 1] *= corr;
      }
      m[r] = mnew;
    }
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = exp2f(s[np][x][i] - m[i >> 1]);  // 0 for keys past N (s = -inf)
          s[np][x][i] = p;
          l[i >> 1] += p;
        }
      uint32_t pa[4];
      c_to_a(pa, s[np]);
      mma_at<D>(o, pa, S.v[st], np * 16);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t j = j0 + jl0 + 8 * r;
    const float il = 1.f / quad_sum(l[r]);  // l >= 1: the max term contributes 2^0
    if (j >= N) continue;
    float* out = a.out_o + (row * N + j) * a.hd + h * a.d;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int e = n * 8 + 2 * (lane & 3) + x;
        if (e < a.d) out[e] = o[n][2 * r + x] * il;
      }
    if (a.out_stat && (lane & 3) == 0) a.out_stat[(row * a.H + h) * N + j] = make_float2(m[r], il);
  }
}

// ---------------------------------------------------------------------------------------
// dq: CTA = (pair row, head, 64 queries); warp = 16 queries; keys in tiles of 64.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) dq_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RowSmem<D>& S = *reinterpret_cast<RowSmem<D>*>(smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int h = blockIdx.y;
  const int64_t row = blockIdx.x, N = a.N, b = row / N;
  const int64_t j0 = static_cast<int64_t>(blockIdx.z) * kRows;
  const __half* kp = plane<D>(a.k, a, row, h);
  const __half* vp = plane<D>(a.v, a, row, h);
  const __half* bp = a.tri + (b * a.H + h) * N * a.Np;
  const float* mrow = mask_row(a, row);
  const int nt = static_cast<int>((N + kRows - 1) / kRows);
  auto issue = [&](int t, int st) {
    const int64_t k0 = static_cast<int64_t>(t) * kRows;
    load_rows<D>(S.k[st], kp, k0, N);
    load_rows<D>(S.v[st], vp, k0, N);
    load_bias(S.b[st], bp, j0, k0, N, a.Np);
    if (threadIdx.x < kRows) S.m[st][threadIdx.x] = mask_bias2(a, mrow, k0 + threadIdx.x);
  };
  load_rows<D>(S.k[1], plane<D>(a.q, a, row, h), j0, N);
  load_rows<D>(S.v[1], plane<D>(a.dO, a, row, h), j0, N);
  issue(0, 0);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  uint32_t qf[D / 16][4], gf[D / 16][4];
  load_a<D>(qf, S.k[1], w * 16);
  load_a<D>(gf, S.v[1], w * 16);
  __syncthreads();
  const int jl0 = w * 16 + (lane >> 2);
  float2 stt[2];
  float ds0[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t j = j0 + jl0 + 8 * r;
    const bool in = j < N;
    stt[r] = in ? a.stat[(row * a.H + h) * N + j] : make_float2(0.f, 0.f);
    ds0[r] = in ? a.dsum[(row * a.H + h) * N + j] * a.gscale : 0.f;
  }
  float acc[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  for (int t = 0; t < nt; ++t) {
    const int st = t & 1;
    if (t + 1 < nt) issue(t + 1, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      float s[2][4] = {}, dp[2][4] = {};
      mma_abt<D>(s, qf, S.k[st], np * 16);
      mma_abt<D>(dp, gf, S.v[st], np * 16);
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int kl = np * 16 + x * 8 + 2 * (lane & 3);
          const float2 bb = bias_pair(S.b[st], jl0 + 8 * r, kl);
          const float s0 = fmaf(s[x][2 * r], a.qscale, fmaf(bb.x, kLog2e, S.m[st][kl]));
          const float s1 = fmaf(s[x][2 * r + 1], a.qscale, fmaf(bb.y, kLog2e, S.m[st][kl + 1]));
          const float p0 = exp2f(s0 - stt[r].x) * stt[r].y, p1 = exp2f(s1 - stt[r].x) * stt[r].y;
          s[x][2 * r] = p0 * (dp[x][2 * r] - ds0[r]);
          s[x][2 * r + 1] = p1 * (dp[x][2 * r + 1] - ds0[r]);
        }
      uint32_t da[4];
      c_to_a(da, s);
      mma_at<D>(acc, da, S.k[st], np * 16);
    }
    __syncthreads();
  }
  const float sc = a.qscale / (kLog2e * a.gscale);  // 1 / (sqrt(d) gscale)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t j = j0 + jl0 + 8 * r;
    if (j >= N) continue;
    float* out = a.dq + (row * N + j) * a.hd + h * a.d;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int e = n * 8 + 2 * (lane & 3) + x;
        if (e < a.d) out[e] = acc[n][2 * r + x] * sc;
      }
  }
}

// ---------------------------------------------------------------------------------------
// dk, dv: CTA = (pair row, head, 64 keys); warp = 16 keys; queries in tiles of 64. The
// products run transposed: S^T = K Q^T, dP^T = V dO^T, dv += P^T dO, dk += dS^T Q.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads) dkv_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ColSmem<D>& S = *reinterpret_cast<ColSmem<D>*>(smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int h = blockIdx.y;
  const int64_t row = blockIdx.x, N = a.N, b = row / N;
  const int64_t k0 = static_cast<int64_t>(blockIdx.z) * kRows;
  const __half* qp = plane<D>(a.q, a, row, h);
  const __half* gp = plane<D>(a.dO, a, row, h);
  const __half* bp = a.tri + (b * a.H + h) * N * a.Np;
  const float2* strow = a.stat + (row * a.H + h) * N;
  const float* dsrow = a.dsum + (row * a.H + h) * N;
  const int nt = static_cast<int>((N + kRows - 1) / kRows);
  auto issue = [&](int t, int st) {
    const int64_t j0 = static_cast<int64_t>(t) * kRows;
    load_rows<D>(S.q[st], qp, j0, N);
    load_rows<D>(S.g[st], gp, j0, N);
    load_bias(S.b[st], bp, j0, k0, N, a.Np);
    if (threadIdx.x < kRows) {
      const int64_t j = j0 + threadIdx.x;
      // past the last query: 1 / l = 0 makes p = 0 (the score there is finite or -inf)
      S.l[st][threadIdx.x] = j < N ? strow[j] : make_float2(0.f, 0.f);
      S.dsum[st][threadIdx.x] = j < N ? dsrow[j] * a.gscale : 0.f;
    }
  };
  load_rows<D>(S.q[1], plane<D>(a.k, a, row, h), k0, N);
  load_rows<D>(S.g[1], plane<D>(a.v, a, row, h), k0, N);
  issue(0, 0);
  cp_commit();
  cp_wait<0>();
  __syncthreads();
  uint32_t kf[D / 16][4], vf[D / 16][4];
  load_a<D>(kf, S.q[1], w * 16);
  load_a<D>(vf, S.g[1], w * 16);
  __syncthreads();
  const int kl0 = w * 16 + (lane >> 2);  // this thread's keys: kl0 and kl0 + 8 of the CTA's 64
  float mb[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) mb[r] = mask_bias2(a, mask_row(a, row), k0 + kl0 + 8 * r);  // -inf past N: p = 0
  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    dk[n][0] = dk[n][1] = dk[n][2] = dk[n][3] = 0.f;
    dv[n][0] = dv[n][1] = dv[n][2] = dv[n][3] = 0.f;
  }
  for (int t = 0; t < nt; ++t) {
    const int st = t & 1;
    if (t + 1 < nt) issue(t + 1, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      float s[2][4] = {}, dp[2][4] = {}, ds[2][4];
      mma_abt<D>(s, kf, S.q[st], np * 16);
      mma_abt<D>(dp, vf, S.g[st], np * 16);
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = i >> 1;
          const int jl = np * 16 + x * 8 + c_col(i);
          const float bb = __half2float(S.b[st][jl][kl0 + 8 * r]);
          const float2 L = S.l[st][jl];
          const float p = exp2f(fmaf(s[x][i], a.qscale, fmaf(bb, kLog2e, mb[r])) - L.x) * L.y;
          s[x][i] = p;
          ds[x][i] = p * (dp[x][i] - S.dsum[st][jl]);
        }
      uint32_t pa[4], da[4];
      c_to_a(pa, s);
      c_to_a(da, ds);
      mma_at<D>(dv, pa, S.g[st], np * 16);
      mma_at<D>(dk, da, S.q[st], np * 16);
    }
    __syncthreads();
  }
  const float sk = a.qscale / (kLog2e * a.gscale), sv = 1.f / a.gscale;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t k = k0 + kl0 + 8 * r;
    if (k >= N) continue;
    const int64_t o = (row * N + k) * a.hd + h * a.d;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int e = n * 8 + 2 * (lane & 3) + x;
        if (e < a.d) {
          a.dk[o + e] = dk[n][2 * r + x] * sk;
          a.dv[o + e] = dv[n][2 * r + x] * sv;
        }
      }
  }
}

// ---------------------------------------------------------------------------------------
// dtri[b,h,j,k] = sum_i ds[i,h,j,k]: CTA = (b*H + h, 64 queries j, 64 keys k), warp = 16
// queries; loops over the pair rows i with that row's q, do, k, v tiles double buffered.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads, D <= 32 ? 4 : 2) dtri_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TriSmem<D>& S = *reinterpret_cast<TriSmem<D>*>(smem_raw);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t bh = blockIdx.x, N = a.N;
  const int64_t b = bh / a.H;
  const int h = static_cast<int>(bh - b * a.H);
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * kRows;
  const int64_t k0 = static_cast<int64_t>(blockIdx.z) * kRows;
  const int jl0 = w * 16 + (lane >> 2);
  auto issue = [&](int64_t i, int st) {
    const int64_t row = b * N + i;
    load_rows<D>(S.q[st], plane<D>(a.q, a, row, h), j0, N);
    load_rows<D>(S.g[st], plane<D>(a.dO, a, row, h), j0, N);
    load_rows<D>(S.k[st], plane<D>(a.k, a, row, h), k0, N);
    load_rows<D>(S.v[st], plane<D>(a.v, a, row, h), k0, N);
    if (threadIdx.x < kRows) {
      const int t = threadIdx.x;
      const int64_t j = j0 + t;
      S.m[st][t] = mask_bias2(a, mask_row(a, row), k0 + t);
      S.l[st][t] = j < N ? a.stat[(row * a.H + h) * N + j] : make_float2(0.f, 0.f);
      S.dsum[st][t] = j < N ? a.dsum[(row * a.H + h) * N + j] * a.gscale : 0.f;
    }
  };
  // the bias block (zero past N) rides with the first row's tiles; kept in shared memory so
  // that registers allow four CTAs per SM
  load_bias(S.bias, a.tri + bh * N * a.Np, j0, k0, N, a.Np);
  issue(0, 0);
  cp_commit();
  float acc[4][2][4];
#pragma unroll
  for (int np = 0; np < 4; ++np)
#pragma unroll
    for (int x = 0; x < 2; ++x) acc[np][x][0] = acc[np][x][1] = acc[np][x][2] = acc[np][x][3] = 0.f;
  for (int64_t i = 0; i < N; ++i) {
    const int st = static_cast<int>(i & 1);
    if (i + 1 < N) issue(i + 1, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    uint32_t qf[D / 16][4], gf[D / 16][4];
    load_a<D>(qf, S.q[st], w * 16);
    load_a<D>(gf, S.g[st], w * 16);
    float2 L[2];
    float d0[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      L[r] = S.l[st][jl0 + 8 * r];
      d0[r] = S.dsum[st][jl0 + 8 * r];
    }
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      float s[2][4] = {}, dp[2][4] = {};
      mma_abt<D>(s, qf, S.k[st], np * 16);
      mma_abt<D>(dp, gf, S.v[st], np * 16);
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int kl = np * 16 + x * 8 + 2 * (lane & 3);
          const float2 bb = bias_pair(S.bias, jl0 + 8 * r, kl);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int e = 2 * r + u;
            const float mk = S.m[st][kl + u];
            const float p = exp2f(fmaf(s[x][e], a.qscale, fmaf(u ? bb.y : bb.x, kLog2e, mk)) - L[r].x) * L[r].y;
            acc[np][x][e] = fmaf(p, dp[x][e] - d0[r], acc[np][x][e]);
          }
        }
    }
    __syncthreads();
  }
  const float sc = 1.f / a.gscale;
#pragma unroll
  for (int np = 0; np < 4; ++np)
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t j = j0 + jl0 + 8 * (e >> 1), k = k0 + np * 16 + x * 8 + c_col(e);
        if (j < N && k < N) a.dtri[(bh * N + j) * N + k] = acc[np][x][e] * sc;
      }
}

// ---------------------------------------------------------------------------------------
// Packing: fp32 [B*N rows][N][H*d] -> fp16 [B*N][H][N][Dp] times `scale`, zero past d; and
// the bias fp32 [B*H][N][N] -> fp16 [B*H][N][Np], zero past N. Eight halves per thread.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    pack_rows_kernel(const float* __restrict__ src, int64_t ld, int64_t rows, int64_t N, int H, int d, int Dp,
                     float scale, __half* __restrict__ dst, uint32_t* status) {
  const int C = Dp / 8;
  const int64_t total = rows * H * N * C;
  uint32_t sat = 0;  // a value beyond the fp16 range was clamped
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % C);
    int64_t rest = idx / C;
    const int64_t j = rest % N;
    rest /= N;
    const int h = static_cast<int>(rest % H);
    const int64_t row = rest / H;
    const float* s = src + (row * N + j) * ld + static_cast<int64_t>(h) * d;
    __align__(16) __half v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = c * 8 + u;
      v[u] = f16_sat_chk(e < d ? s[e] * scale : 0.f, sat);
    }
    *reinterpret_cast<uint4*>(dst + idx * 8) = *reinterpret_cast<const uint4*>(v);
  }
  flag_saturation(sat, status);
}

__global__ void __launch_bounds__(256)
    pack_bias_kernel(const float* __restrict__ src, int64_t planes_rows, int64_t N, int64_t Np,
                     __half* __restrict__ dst) {
  const int64_t C = Np / 8;
  const int64_t total = planes_rows * C;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / C, c = idx - r * C;
    const float* s = src + r * N;
    __align__(16) __half v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t k = c * 8 + u;
      v[u] = __float2half_rn(k < N ? s[k] : 0.f);
    }
    *reinterpret_cast<uint4*>(dst + idx * 8) = *reinterpret_cast<const uint4*>(v);
  }
}

// A tile of 64 rows x D fp16 values staged from fp32 (the generic attention core below).
template <int D>
struct Tile {
  __half v[kRows][D + 8];
};

// Rows r0 .. r0+63 of a row-major fp32 matrix (row pitch ld, `valid` rows in all, the head's
// first column already applied to src) into a tile, times `scale`; zero past d and past the
// last row.
template <int D>
__device__ __forceinline__ void stage(Tile<D>& t, const float* __restrict__ src, int64_t r0, int64_t valid, int d,
                                      int64_t ld, float scale) {
  for (int idx = threadIdx.x; idx < kRows * (D / 2); idx += kThreads) {
    const int r = idx / (D / 2), e = (idx - r * (D / 2)) * 2;
    float x0 = 0.f, x1 = 0.f;
    if (r0 + r < valid) {
      const float* p = src + (r0 + r) * ld + e;
      if (e < d) x0 = p[0] * scale;
      if (e + 1 < d) x1 = p[1] * scale;
    }
    *reinterpret_cast<__half2*>(&t.v[r][e]) = __floats2half2_rn(x0, x1);
  }
}

// ---------------------------------------------------------------------------------------
// Generic gated multi-head attention core (reference primitives.py:114-178 without the
// projections): o[l, q, h] = softmax_k(scale q[l,q,h].k[l,k,h] + bias0 + bias1) v[l, k, h].
// q [L, Q, H*d], k, v [L, K, H*d], o [L, Q, H*d], fp32. Each bias is optional and read
// through five element strides over (l0, l1, h, q, k), l = l0 * L1 + l1 -- a zero stride
// broadcasts, so the reference's [*, 1, 1, K] mask biases and [*, H, Q, K] pair biases are
// read in place. CTA = (l, head, 64 queries), warp = 16 queries.
// ---------------------------------------------------------------------------------------
struct Bias {
  const float* p;
  int64_t s[5];
};

struct MhaArgs {
  const float* q;
  const float* k;
  const float* v;
  Bias bias[2];
  float* o;
  int64_t L1, Q, K;
  int H, d, hd;
  float qscale;  // scale * log2 e
};

__device__ __forceinline__ float bias_at(const Bias& bb, int64_t l0, int64_t l1, int h, int64_t q, int64_t k) {
  return bb.p[l0 * bb.s[0] + l1 * bb.s[1] + h * bb.s[2] + q * bb.s[3] + k * bb.s[4]];
}

template <int D>
__global__ void __launch_bounds__(kThreads) mha_fwd_kernel(const MhaArgs a) {
  __shared__ __align__(16) Tile<D> Ks, Vs;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int h = blockIdx.y;
  const int64_t l = blockIdx.x, l0 = l / a.L1, l1 = l - l0 * a.L1;
  const int64_t Q = a.Q, K = a.K;
  const int64_t q0 = static_cast<int64_t>(blockIdx.z) * kRows;
  const float* rk = a.k + l * K * a.hd + h * a.d;
  const float* rv = a.v + l * K * a.hd + h * a.d;
  stage<D>(Ks, a.q + l * Q * a.hd + h * a.d, q0, Q, a.d, a.hd, a.qscale);
  __syncthreads();
  uint32_t qf[D / 16][4];
  load_a<D>(qf, Ks.v, w * 16);
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, ls[2] = {0.f, 0.f};
  int64_t qr[2];
  qr[0] = q0 + w * 16 + (lane >> 2);
  qr[1] = qr[0] + 8;
  for (int64_t k0 = 0; k0 < K; k0 += kRows) {
    __syncthreads();
    stage<D>(Ks, rk, k0, K, a.d, a.hd, 1.f);
    stage<D>(Vs, rv, k0, K, a.d, a.hd, 1.f);
    __syncthreads();
    float s[4][2][4];
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int x = 0; x < 2; ++x) s[np][x][0] = s[np][x][1] = s[np][x][2] = s[np][x][3] = 0.f;
      mma_abt<D>(s[np], qf, Ks.v, np * 16);
    }
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int np = 0; np < 4; ++np)
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int64_t k = k0 + np * 16 + x * 8 + c_col(i), qq = qr[i >> 1];
          float bias = -INFINITY;
          if (k < K) {
            bias = 0.f;
            if (qq < Q) {
#pragma unroll
              for (int t = 0; t < 2; ++t)
                if (a.bias[t].p) bias += bias_at(a.bias[t], l0, l1, h, qq, k);
              bias *= kLog2e;
            }
          }
          s[np][x][i] += bias;
          tmax[i >> 1] = fmaxf(tmax[i >> 1], s[np][x][i]);
        }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float mnew = fmaxf(m[r], quad_max(tmax[r]));
      // a row whose scores are all -inf so far keeps m = -inf: guard the rescale
      const float corr = mnew == -INFINITY ? 1.f : exp2f(m[r] - mnew);
      ls[r] *= corr;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        o[n][2 * r] *= corr;
        o[n][2 * r + 1] *= corr;
      }
      m[r] = mnew;
    }
#pragma unroll
    for (int np = 0; np < 4; ++np) {
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float mr = m[i >> 1];
          const float p = mr == -INFINITY ? 0.f : exp2f(s[np][x][i] - mr);
          s[np][x][i] = p;
          ls[i >> 1] += p;
        }
      uint32_t pa[4];
      c_to_a(pa, s[np]);
      mma_at<D>(o, pa, Vs.v, np * 16);
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const float lsum = quad_sum(ls[r]);
    if (qr[r] >= Q) continue;
    // every score -inf (a bias of -inf on every key): softmax is NaN in the reference too
    const float il = lsum > 0.f ? 1.f / lsum : NAN;
    float* out = a.o + (l * Q + qr[r]) * a.hd + h * a.d;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int e = n * 8 + 2 * (lane & 3) + x;
        if (e < a.d) out[e] = o[n][2 * r + x] * il;
      }
  }
}

static int check_core(const Args& a, int64_t B) {
  if (B < 1 || a.N < 1 || B * a.N > 2147483647 || (a.N + kRows - 1) / kRows > 65535)
    return fail(GTK_ERR_INVALID_ARG, "attention core: bad B / N");
  if (a.H < 1 || a.H > 65535 || a.d < 1 || a.d > 64 || a.hd != a.H * a.d)
    return fail(GTK_ERR_UNSUPPORTED, "attention core: need 1 <= heads and 1 <= head_dim <= 64");
  if (!(std::isfinite(a.inf2))) return fail(GTK_ERR_INVALID_ARG, "attention core: inf must be finite");
  return GTK_OK;
}

static int padded_dim(int d) { return d <= 16 ? 16 : (d <= 32 ? 32 : 64); }

static Args core_args(int64_t N, int heads, int head_dim, float inf) {
  Args a{};
  a.N = N;
  a.Np = (N + 7) / 8 * 8;
  a.msi = N;
  a.msk = 1;
  a.H = heads;
  a.d = head_dim;
  a.hd = heads * head_dim;
  a.qscale = kLog2e / std::sqrt(static_cast<float>(head_dim > 0 ? head_dim : 1));
  a.inf2 = inf * kLog2e;
  a.gscale = 1.f;
  return a;
}

// Launch KERNEL<Dp> with its shared-memory struct SMEM<Dp> (opting in above 48 KB once per
// device).
#define GTK_CORE_LAUNCH(KERNEL, SMEM, GRID, WHAT)                                                     \
  do {                                                                                                 \
    auto go = [&](auto kern, int bytes) -> int {                                                       \
      if (int e = ensure_smem(reinterpret_cast<const void*>(kern), bytes)) return e;                   \
      kern<<<GRID, kThreads, bytes, st>>>(a);                                                          \
      return check_launch(WHAT);                                                                       \
    };                                                                                                 \
    const int dp = padded_dim(a.d);                                                                    \
    const int rc = dp == 16   ? go(KERNEL<16>, static_cast<int>(sizeof(SMEM<16>)))                      \
                   : dp == 32 ? go(KERNEL<32>, static_cast<int>(sizeof(SMEM<32>)))                      \
                              : go(KERNEL<64>, static_cast<int>(sizeof(SMEM<64>)));                     \
    if (rc) return rc;                                                                                 \
  } while (0)

#define GTK_ATTN_LAUNCH(KERNEL, GRID, ARGS, HEAD_DIM)                          \
  do {                                                                         \
    if ((HEAD_DIM) <= 16)                                                      \
      KERNEL<16><<<GRID, kThreads, 0, st>>>(ARGS);                             \
    else if ((HEAD_DIM) <= 32)                                                 \
      KERNEL<32><<<GRID, kThreads, 0, st>>>(ARGS);                             \
    else                                                                       \
      KERNEL<64><<<GRID, kThreads, 0, st>>>(ARGS);                             \
  } while (0)

static unsigned grid_1d(int64_t work, int per_block) {
  const int64_t need = (work + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  return static_cast<unsigned>(need < 1 ? 1 : (need < cap ? need : cap));
}

int padded_head_dim(int d) { return padded_dim(d); }

int launch_pack(const float* src, int64_t ld, int64_t B, int64_t N, int H, int d, float scale, __half* dst,
                uint32_t* status, cudaStream_t st, int Dp) {
  const int dp = Dp > 0 ? Dp : padded_dim(d);
  if (dp % 8 || dp < d) return fail(GTK_ERR_INVALID_ARG, "attention core pack: bad plane width");
  pack_rows_kernel<<<grid_1d(B * N * H * N * (dp / 8), 256), 256, 0, st>>>(src, ld, B * N, N, H, d, dp, scale, dst,
                                                                          status);
  return check_launch("attention core pack");
}

int launch_forward(const __half* q, const __half* k, const __half* v, const __half* tri, const float* mask,
                   int64_t msi, int64_t msk, int64_t B, int64_t N, int H, int d, float inf, float* o,
                   cudaStream_t st) {
  Args a = core_args(N, H, d, inf);
  a.q = q;
  a.k = k;
  a.v = v;
  a.tri = tri;
  a.mask = mask;
  a.msi = msi;
  a.msk = msk;
  a.out_o = o;
  if (int e = check_core(a, B)) return e;
  const dim3 grid(static_cast<unsigned>(B * N), static_cast<unsigned>(H), static_cast<unsigned>((N + kRows - 1) / kRows));
  GTK_CORE_LAUNCH(fwd_kernel, RowSmem, grid, "attention core forward");
  return GTK_OK;
}

}  // namespace attn
}  // namespace gtk

using namespace gtk;
using namespace gtk::attn;

extern "C" {

size_t gtk_attn_core_packed_bytes(int64_t B, int64_t N, int heads, int head_dim) {
  if (B < 1 || N < 1 || heads < 1 || head_dim < 1 || head_dim > 64) return 0;
  return static_cast<size_t>(B) * N * heads * N * padded_dim(head_dim) * 2;
}

size_t gtk_attn_core_bias_bytes(int64_t B, int64_t N, int heads) {
  if (B < 1 || N < 1 || heads < 1) return 0;
  return static_cast<size_t>(B) * heads * N * ((N + 7) / 8 * 8) * 2;
}

int gtk_attn_core_pack(const float* src, int64_t B, int64_t N, int heads, int head_dim, float scale, void* dst,
                       void* stream) {
  if (B < 1 || N < 1 || !dims_ok(B * N) || heads < 1 || heads > 65535 || head_dim < 1 || head_dim > 64)
    return fail(GTK_ERR_INVALID_ARG, "attention core pack: bad sizes (head_dim <= 64)");
  if (!std::isfinite(scale)) return fail(GTK_ERR_INVALID_ARG, "attention core pack: scale must be finite");
  if (int e = check_ptr(src, "src", 4)) return e;
  if (int e = check_ptr(dst, "dst", 16)) return e;
  if (int e = check_device()) return e;
  const int dp = padded_dim(head_dim);
  const int64_t work = B * N * heads * N * (dp / 8);
  pack_rows_kernel<<<grid_1d(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, static_cast<int64_t>(heads) * head_dim, B * N, N, heads, head_dim, dp, scale, static_cast<__half*>(dst),
      nullptr);
  return check_launch("attention core pack");
}

int gtk_attn_core_pack_bias(const float* tri, int64_t B, int64_t N, int heads, void* dst, void* stream) {
  if (B < 1 || N < 1 || heads < 1 || !dims_ok(B * heads * N)) return fail(GTK_ERR_INVALID_ARG, "bias pack: bad sizes");
  if (int e = check_ptr(tri, "tri", 4)) return e;
  if (int e = check_ptr(dst, "dst", 16)) return e;
  if (int e = check_device()) return e;
  const int64_t Np = (N + 7) / 8 * 8;
  pack_bias_kernel<<<grid_1d(B * heads * N * (Np / 8), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      tri, B * heads * N, N, Np, static_cast<__half*>(dst));
  return check_launch("attention core bias pack");
}

int gtk_attn_core_forward(const void* q, const void* k, const void* v, const void* tri, const float* mask, int64_t B,
                          int64_t N, int heads, int head_dim, float inf, float* o, float* stats, void* stream) {
  Args a = core_args(N, heads, head_dim, inf);
  a.q = static_cast<const __half*>(q);
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.tri = static_cast<const __half*>(tri);
  a.mask = mask;
  a.out_o = o;
  a.out_stat = reinterpret_cast<float2*>(stats);
  if (int e = check_core(a, B)) return e;
  for (const void* p : {q, k, v, tri})
    if (int e = check_ptr(p, "packed attention operand", 16)) return e;
  if (int e = check_ptr(o, "o", 4)) return e;
  if (int e = check_ptr(stats, "stats", 8)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (int e = check_device()) return e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(B * N), static_cast<unsigned>(heads),
                  static_cast<unsigned>((N + kRows - 1) / kRows));
  GTK_CORE_LAUNCH(fwd_kernel, RowSmem, grid, "attention core forward");
  return GTK_OK;
}

int gtk_attn_core_backward(const void* q, const void* k, const void* v, const void* tri, const float* mask,
                           const float* stats, const void* dO, const float* dsum, float dO_scale, int64_t B, int64_t N,
                           int heads, int head_dim, float inf, float* dq, float* dk, float* dv, float* dtri,
                           void* stream) {
  Args a = core_args(N, heads, head_dim, inf);
  a.q = static_cast<const __half*>(q);
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.tri = static_cast<const __half*>(tri);
  a.mask = mask;
  a.stat = reinterpret_cast<const float2*>(stats);
  a.dO = static_cast<const __half*>(dO);
  a.dsum = dsum;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.dtri = dtri;
  a.gscale = dO_scale;
  if (int e = check_core(a, B)) return e;
  if (!(dO_scale > 0.f) || !std::isfinite(dO_scale))
    return fail(GTK_ERR_INVALID_ARG, "attention core: dO_scale must be finite and > 0");
  if (B * heads > 2147483647) return fail(GTK_ERR_INVALID_ARG, "attention core: B * heads too large");
  for (const void* p : {q, k, v, tri, dO})
    if (int e = check_ptr(p, "packed attention operand", 16)) return e;
  for (const void* p : {static_cast<const void*>(dsum), static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv), static_cast<const void*>(dtri)})
    if (int e = check_ptr(p, "attention core tensor", 4)) return e;
  if (int e = check_ptr(stats, "stats", 8)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (int e = check_device()) return e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned nb = static_cast<unsigned>((N + kRows - 1) / kRows);
  const dim3 rows(static_cast<unsigned>(B * N), static_cast<unsigned>(heads), nb);
  GTK_CORE_LAUNCH(dq_kernel, RowSmem, rows, "attention core backward (dq)");
  GTK_CORE_LAUNCH(dkv_kernel, ColSmem, rows, "attention core backward (dk, dv)");
  const dim3 bias(static_cast<unsigned>(B * heads), nb, nb);
  GTK_CORE_LAUNCH(dtri_kernel, TriSmem, bias, "attention core backward (dtri)");
  return GTK_OK;
}

int gtk_mha_forward(const float* q, const float* k, const float* v, const float* bias0, const int64_t* strides0,
                    const float* bias1, const int64_t* strides1, int64_t L0, int64_t L1, int64_t Q, int64_t K,
                    int heads, int head_dim, float scale, float* o, void* stream) {
  if (L0 < 1 || L1 < 1 || Q < 1 || K < 1 || L0 * L1 > 2147483647 || (Q + kRows - 1) / kRows > 65535)
    return fail(GTK_ERR_INVALID_ARG, "mha: bad batch / length");
  if (heads < 1 || heads > 65535 || head_dim < 1 || head_dim > 64)
    return fail(GTK_ERR_UNSUPPORTED, "mha: need 1 <= heads and 1 <= head_dim <= 64");
  if (!std::isfinite(scale)) return fail(GTK_ERR_INVALID_ARG, "mha: scale must be finite");
  for (const void* p : {static_cast<const void*>(q), static_cast<const void*>(k), static_cast<const void*>(v),
                        static_cast<const void*>(o)})
    if (int e = check_ptr(p, "mha tensor", 4)) return e;
  MhaArgs a{};
  const float* bp[2] = {bias0, bias1};
  const int64_t* bs[2] = {strides0, strides1};
  for (int t = 0; t < 2; ++t) {
    a.bias[t].p = bp[t];
    if (!bp[t]) continue;
    if (!bs[t]) return fail(GTK_ERR_INVALID_ARG, "mha: a bias needs its five strides");
    if (reinterpret_cast<uintptr_t>(bp[t]) & 3) return fail(GTK_ERR_ALIGNMENT, "mha: bias is misaligned");
    for (int x = 0; x < 5; ++x) {
      if (bs[t][x] < 0) return fail(GTK_ERR_INVALID_ARG, "mha: bias strides must be >= 0");
      a.bias[t].s[x] = bs[t][x];
    }
  }
  a.q = q;
  a.k = k;
  a.v = v;
  a.o = o;
  a.L1 = L1;
  a.Q = Q;
  a.K = K;
  a.H = heads;
  a.d = head_dim;
  a.hd = heads * head_dim;
  a.qscale = scale * kLog2e;
  if (int e = check_device()) return e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(L0 * L1), static_cast<unsigned>(heads),
                  static_cast<unsigned>((Q + kRows - 1) / kRows));
  GTK_ATTN_LAUNCH(mha_fwd_kernel, grid, a, head_dim);
  return check_launch("mha forward");
}

}  // extern "C"
