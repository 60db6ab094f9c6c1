// The triangle-attention core for training: forward with the softmax statistics, and its
// backward, without ever forming the [B, N, H, N, N] score tensor.
//
// Frame of the block (z itself for the starting node, z^T for the ending node), pair row i,
// query j, key k, head h, head_dim d (reference primitives.py:134-164):
//   s[i,h,j,k] = q[i,j,h] . k[i,k,h] / sqrt(d) + inf * (m[i,k] - 1) + tri[h,j,k]
//   p = softmax_k(s),  o[i,j,h] = sum_k p v[i,k,h]
// Inputs q, k, v, o and their gradients are fp32 [B, N(i), N(j), H*d] (the layout of the
// projections), tri and its gradient fp32 [B, H, N(j), N(k)], the mask fp32 [B, N(i), N(k)]
// in the block's frame (or NULL). The statistics are, per (b, i, h, j), the running max m of
// the base-2 scores and 1 / l, l = sum_k 2^(s2 - m), kept apart: for a fully masked row every
// score is about -1.4e9, and m + log2 l would round back to m.
// With D = sum_e do o per (i, j, h) and ds = p (do . v_k - D):
//   dq[i,j] = sum_k ds k[i,k] / sqrt(d)      (query-major kernel, thread = query)
//   dk[i,k] = sum_j ds q[i,j] / sqrt(d),  dv[i,k] = sum_j p do[i,j]   (key-major, thread = key)
//   dtri[h,j,k] = sum_i ds[i,h,j,k]          (bias-major: CTA = query block x key block, loop over i)
// Everything is fp32 on the CUDA cores; softmax in base 2 (scores and bias carry log2 e).
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQ = 128;   // queries (or keys) per CTA, one per thread
constexpr int kT = 32;    // keys (or queries) per shared-memory tile

struct Args {
  const float* q;
  const float* k;
  const float* v;
  const float* tri;
  const float* mask;
  const float* o;
  const float2* stat;  // (m, 1 / l) per [b][i][h][j]
  const float* dO;
  const float* dsum;   // D[b][i][h][j]
  float* out_o;
  float2* out_stat;
  float* dq;
  float* dk;
  float* dv;
  float* dtri;
  int64_t N;
  int H, d, hd;
  float qscale;  // log2 e / sqrt(d)
  float inf2;    // inf * log2 e
};

__device__ __forceinline__ float mask_bias2(const Args& a, int64_t row, int64_t k) {
  if (k >= a.N) return -INFINITY;
  return a.mask ? a.inf2 * (a.mask[row * a.N + k] - 1.f) : 0.f;
}

// ---------------------------------------------------------------------------------------
// Forward with statistics. CTA = (row b*N+i, head h, 128 queries); thread = query.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kQ) fwd_kernel(const Args a) {
  __shared__ float Ks[kT][D], Vs[kT][D];
  __shared__ float Bs[kQ][kT + 1];
  __shared__ float Ms[kT];
  const int t = threadIdx.x, h = blockIdx.y;
  const int64_t row = blockIdx.x, N = a.N;
  const int64_t b = row / N;
  const int64_t j0 = static_cast<int64_t>(blockIdx.z) * kQ, j = j0 + t;
  const bool active = j < N;
  float q[D], o[D];
  const float* yq = a.q + (row * N + (active ? j : 0)) * a.hd + h * a.d;
#pragma unroll
  for (int e = 0; e < D; ++e) {
    q[e] = (e < a.d && active) ? yq[e] * a.qscale : 0.f;
    o[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const float* trib = a.tri + (b * a.H + h) * N * N;
  for (int64_t k0 = 0; k0 < N; k0 += kT) {
    __syncthreads();
    for (int idx = t; idx < kT * D; idx += kQ) {
      const int kk = idx / D, e = idx - kk * D;
      const int64_t k = k0 + kk;
      const bool in = k < N && e < a.d;
      Ks[kk][e] = in ? a.k[(row * N + k) * a.hd + h * a.d + e] : 0.f;
      Vs[kk][e] = in ? a.v[(row * N + k) * a.hd + h * a.d + e] : 0.f;
    }
    for (int idx = t; idx < kQ * kT; idx += kQ) {
      const int jj = idx / kT, kk = idx - jj * kT;
      const int64_t jq = j0 + jj, k = k0 + kk;
      Bs[jj][kk] = (jq < N && k < N) ? trib[jq * N + k] * kLog2e : 0.f;
    }
    if (t < kT) Ms[t] = mask_bias2(a, row, k0 + t);
    __syncthreads();
    float s[kT];
    float tmax = -INFINITY;
#pragma unroll
    for (int kk = 0; kk < kT; ++kk) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < D; ++e) acc = fmaf(q[e], Ks[kk][e], acc);
      s[kk] = acc + Bs[t][kk] + Ms[kk];
      tmax = fmaxf(tmax, s[kk]);
    }
    const float mnew = fmaxf(m, tmax);
    const float corr = exp2f(m - mnew);
    l *= corr;
#pragma unroll
    for (int e = 0; e < D; ++e) o[e] *= corr;
#pragma unroll
    for (int kk = 0; kk < kT; ++kk) {
      const float p = exp2f(s[kk] - mnew);
      l += p;
#pragma unroll
      for (int e = 0; e < D; ++e) o[e] = fmaf(p, Vs[kk][e], o[e]);
    }
    m = mnew;
  }
  if (active) {
    float* out = a.out_o + (row * N + j) * a.hd + h * a.d;
    const float il = 1.f / l;  // l >= 1: the max term contributes 2^0
#pragma unroll
    for (int e = 0; e < D; ++e)
      if (e < a.d) out[e] = o[e] * il;
    a.out_stat[(row * a.H + h) * N + j] = make_float2(m, il);
  }
}

// ---------------------------------------------------------------------------------------
// dq: CTA = (row, head, 128 queries), thread = query; keys in shared-memory tiles.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kQ) dq_kernel(const Args a) {
  __shared__ float Ks[kT][D], Vs[kT][D];
  __shared__ float Bs[kQ][kT + 1];
  __shared__ float Ms[kT];
  const int t = threadIdx.x, h = blockIdx.y;
  const int64_t row = blockIdx.x, N = a.N;
  const int64_t b = row / N;
  const int64_t j0 = static_cast<int64_t>(blockIdx.z) * kQ, j = j0 + t;
  const bool active = j < N;
  const int64_t pj = (row * N + (active ? j : 0)) * a.hd + h * a.d;
  float q[D], g[D], dq[D];
#pragma unroll
  for (int e = 0; e < D; ++e) {
    q[e] = (e < a.d && active) ? a.q[pj + e] * a.qscale : 0.f;
    g[e] = (e < a.d && active) ? a.dO[pj + e] : 0.f;
    dq[e] = 0.f;
  }
  const float2 st = active ? a.stat[(row * a.H + h) * N + j] : make_float2(0.f, 0.f);
  const float dsum = active ? a.dsum[(row * a.H + h) * N + j] : 0.f;
  const float* trib = a.tri + (b * a.H + h) * N * N;
  for (int64_t k0 = 0; k0 < N; k0 += kT) {
    __syncthreads();
    for (int idx = t; idx < kT * D; idx += kQ) {
      const int kk = idx / D, e = idx - kk * D;
      const int64_t k = k0 + kk;
      const bool in = k < N && e < a.d;
      Ks[kk][e] = in ? a.k[(row * N + k) * a.hd + h * a.d + e] : 0.f;
      Vs[kk][e] = in ? a.v[(row * N + k) * a.hd + h * a.d + e] : 0.f;
    }
    for (int idx = t; idx < kQ * kT; idx += kQ) {
      const int jj = idx / kT, kk = idx - jj * kT;
      const int64_t jq = j0 + jj, k = k0 + kk;
      Bs[jj][kk] = (jq < N && k < N) ? trib[jq * N + k] * kLog2e : 0.f;
    }
    if (t < kT) Ms[t] = mask_bias2(a, row, k0 + t);
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kT; ++kk) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int e = 0; e < D; ++e) {
        s = fmaf(q[e], Ks[kk][e], s);
        dp = fmaf(g[e], Vs[kk][e], dp);
      }
      const float p = exp2f(s + Bs[t][kk] + Ms[kk] - st.x) * st.y;
      const float ds = p * (dp - dsum);
#pragma unroll
      for (int e = 0; e < D; ++e) dq[e] = fmaf(ds, Ks[kk][e], dq[e]);
    }
  }
  if (active) {
    const float sc = a.qscale / kLog2e;  // 1 / sqrt(d)
#pragma unroll
    for (int e = 0; e < D; ++e)
      if (e < a.d) a.dq[pj + e] = dq[e] * sc;
  }
}

// ---------------------------------------------------------------------------------------
// dk, dv: CTA = (row, head, 128 keys), thread = key; queries in shared-memory tiles.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kQ) dkv_kernel(const Args a) {
  __shared__ float Qs[kT][D], Gs[kT][D];
  __shared__ float Bs[kT][kQ + 1];
  __shared__ float2 Ls[kT];
  __shared__ float Ds[kT];
  const int t = threadIdx.x, h = blockIdx.y;
  const int64_t row = blockIdx.x, N = a.N;
  const int64_t b = row / N;
  const int64_t k0 = static_cast<int64_t>(blockIdx.z) * kQ, k = k0 + t;
  const bool active = k < N;
  const int64_t pk = (row * N + (active ? k : 0)) * a.hd + h * a.d;
  float kv[D], vv[D], dk[D], dv[D];
#pragma unroll
  for (int e = 0; e < D; ++e) {
    kv[e] = (e < a.d && active) ? a.k[pk + e] : 0.f;
    vv[e] = (e < a.d && active) ? a.v[pk + e] : 0.f;
    dk[e] = 0.f;
    dv[e] = 0.f;
  }
  const float mb = active ? mask_bias2(a, row, k) : -INFINITY;
  const float* trib = a.tri + (b * a.H + h) * N * N;
  for (int64_t j0 = 0; j0 < N; j0 += kT) {
    __syncthreads();
    for (int idx = t; idx < kT * D; idx += kQ) {
      const int jj = idx / D, e = idx - jj * D;
      const int64_t j = j0 + jj;
      const bool in = j < N && e < a.d;
      Qs[jj][e] = in ? a.q[(row * N + j) * a.hd + h * a.d + e] * a.qscale : 0.f;
      Gs[jj][e] = in ? a.dO[(row * N + j) * a.hd + h * a.d + e] : 0.f;
    }
    for (int idx = t; idx < kT * kQ; idx += kQ) {
      const int jj = idx / kQ, kk = idx - jj * kQ;
      const int64_t j = j0 + jj, kq = k0 + kk;
      Bs[jj][kk] = (j < N && kq < N) ? trib[j * N + kq] * kLog2e : 0.f;
    }
    if (t < kT) {
      const int64_t j = j0 + t;
      Ls[t] = j < N ? a.stat[(row * a.H + h) * N + j] : make_float2(0.f, 0.f);  // past the last query: p = 0
      Ds[t] = j < N ? a.dsum[(row * a.H + h) * N + j] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < kT; ++jj) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int e = 0; e < D; ++e) {
        s = fmaf(Qs[jj][e], kv[e], s);
        dp = fmaf(Gs[jj][e], vv[e], dp);
      }
      const float p = exp2f(s + Bs[jj][t] + mb - Ls[jj].x) * Ls[jj].y;
      const float ds = p * (dp - Ds[jj]);
#pragma unroll
      for (int e = 0; e < D; ++e) {
        dk[e] = fmaf(ds, Qs[jj][e], dk[e]);
        dv[e] = fmaf(p, Gs[jj][e], dv[e]);
      }
    }
  }
  if (active) {
    // Qs carried log2 e / sqrt(d): dk = sum ds q / sqrt(d) = (sum ds Qs) / log2 e
#pragma unroll
    for (int e = 0; e < D; ++e)
      if (e < a.d) {
        a.dk[pk + e] = dk[e] * (1.f / kLog2e);
        a.dv[pk + e] = dv[e];
      }
  }
}

// ---------------------------------------------------------------------------------------
// dtri[h,j,k] = sum_i ds[i,h,j,k]: CTA = (b*H + h, 128 queries j, 32 keys k), thread = query;
// loops over the rows i with that row's 32 keys and values staged in shared memory.
// ---------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kQ) dtri_kernel(const Args a) {
  __shared__ float Ks[kT][D], Vs[kT][D];
  __shared__ float Ms[kT];
  const int t = threadIdx.x;
  const int64_t bh = blockIdx.x, N = a.N;
  const int64_t b = bh / a.H;
  const int h = static_cast<int>(bh - b * a.H);
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * kQ, j = j0 + t;
  const int64_t k0 = static_cast<int64_t>(blockIdx.z) * kT;
  const bool active = j < N;
  float acc[kT];
  float bias[kT];
  const float* trib = a.tri + bh * N * N + (active ? j : 0) * N + k0;
#pragma unroll
  for (int kk = 0; kk < kT; ++kk) {
    acc[kk] = 0.f;
    bias[kk] = (active && k0 + kk < N) ? trib[kk] * kLog2e : 0.f;
  }
  for (int64_t i = 0; i < N; ++i) {
    const int64_t row = b * N + i;
    __syncthreads();
    for (int idx = t; idx < kT * D; idx += kQ) {
      const int kk = idx / D, e = idx - kk * D;
      const int64_t k = k0 + kk;
      const bool in = k < N && e < a.d;
      Ks[kk][e] = in ? a.k[(row * N + k) * a.hd + h * a.d + e] : 0.f;
      Vs[kk][e] = in ? a.v[(row * N + k) * a.hd + h * a.d + e] : 0.f;
    }
    if (t < kT) Ms[t] = mask_bias2(a, row, k0 + t);
    __syncthreads();
    if (!active) continue;
    const int64_t pj = (row * N + j) * a.hd + h * a.d;
    float q[D], g[D];
#pragma unroll
    for (int e = 0; e < D; ++e) {
      q[e] = e < a.d ? a.q[pj + e] * a.qscale : 0.f;
      g[e] = e < a.d ? a.dO[pj + e] : 0.f;
    }
    const float2 st = a.stat[(row * a.H + h) * N + j];
    const float dsum = a.dsum[(row * a.H + h) * N + j];
#pragma unroll
    for (int kk = 0; kk < kT; ++kk) {
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int e = 0; e < D; ++e) {
        s = fmaf(q[e], Ks[kk][e], s);
        dp = fmaf(g[e], Vs[kk][e], dp);
      }
      const float p = exp2f(s + bias[kk] + Ms[kk] - st.x) * st.y;
      acc[kk] = fmaf(p, dp - dsum, acc[kk]);
    }
  }
  if (active) {
    float* out = a.dtri + bh * N * N + j * N + k0;
#pragma unroll
    for (int kk = 0; kk < kT; ++kk)
      if (k0 + kk < N) out[kk] = acc[kk];
  }
}

static int check(const Args& a, int64_t B) {
  if (B < 1 || a.N < 1 || B * a.N > 2147483647 || (a.N + kQ - 1) / kQ > 65535)
    return fail(GTK_ERR_INVALID_ARG, "attention core: bad B / N");
  if (a.H < 1 || a.H > 65535 || a.d < 1 || a.d > 64 || a.hd != a.H * a.d)
    return fail(GTK_ERR_UNSUPPORTED, "attention core: need 1 <= heads and 1 <= head_dim <= 64");
  if (!(std::isfinite(a.inf2))) return fail(GTK_ERR_INVALID_ARG, "attention core: inf must be finite");
  return GTK_OK;
}

#define GTK_ATTN_LAUNCH(KERNEL, GRID)                                          \
  do {                                                                         \
    if (a.d <= 8)                                                              \
      KERNEL<8><<<GRID, kQ, 0, st>>>(a);                                       \
    else if (a.d <= 16)                                                        \
      KERNEL<16><<<GRID, kQ, 0, st>>>(a);                                      \
    else if (a.d <= 32)                                                        \
      KERNEL<32><<<GRID, kQ, 0, st>>>(a);                                      \
    else                                                                       \
      KERNEL<64><<<GRID, kQ, 0, st>>>(a);                                      \
  } while (0)

}  // namespace attn
}  // namespace gtk

using namespace gtk;
using namespace gtk::attn;

extern "C" {

int gtk_attn_core_forward(const float* q, const float* k, const float* v, const float* tri, const float* mask,
                          int64_t B, int64_t N, int heads, int head_dim, float inf, float* o, float* stats,
                          void* stream) {
  Args a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.tri = tri;
  a.mask = mask;
  a.out_o = o;
  a.out_stat = reinterpret_cast<float2*>(stats);
  a.N = N;
  a.H = heads;
  a.d = head_dim;
  a.hd = heads * head_dim;
  a.qscale = kLog2e / std::sqrt(static_cast<float>(head_dim > 0 ? head_dim : 1));
  a.inf2 = inf * kLog2e;
  if (int e = check(a, B)) return e;
  for (const void* p : {static_cast<const void*>(q), static_cast<const void*>(k), static_cast<const void*>(v),
                        static_cast<const void*>(tri), static_cast<const void*>(o)})
    if (int e = check_ptr(p, "attention core tensor", 4)) return e;
  if (int e = check_ptr(stats, "stats", 8)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (int e = check_device()) return e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(B * N), static_cast<unsigned>(heads), static_cast<unsigned>((N + kQ - 1) / kQ));
  GTK_ATTN_LAUNCH(fwd_kernel, grid);
  return check_launch("attention core forward");
}

int gtk_attn_core_backward(const float* q, const float* k, const float* v, const float* tri, const float* mask,
                           const float* stats, const float* dO, const float* dsum, int64_t B, int64_t N, int heads,
                           int head_dim, float inf, float* dq, float* dk, float* dv, float* dtri, void* stream) {
  Args a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.tri = tri;
  a.mask = mask;
  a.stat = reinterpret_cast<const float2*>(stats);
  a.dO = dO;
  a.dsum = dsum;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.dtri = dtri;
  a.N = N;
  a.H = heads;
  a.d = head_dim;
  a.hd = heads * head_dim;
  a.qscale = kLog2e / std::sqrt(static_cast<float>(head_dim > 0 ? head_dim : 1));
  a.inf2 = inf * kLog2e;
  if (int e = check(a, B)) return e;
  if (B * heads > 2147483647 || (N + kT - 1) / kT > 65535) return fail(GTK_ERR_INVALID_ARG, "attention core: N too large");
  for (const void* p : {static_cast<const void*>(q), static_cast<const void*>(k), static_cast<const void*>(v),
                        static_cast<const void*>(tri), static_cast<const void*>(dO),
                        static_cast<const void*>(dsum), static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv), static_cast<const void*>(dtri)})
    if (int e = check_ptr(p, "attention core tensor", 4)) return e;
  if (int e = check_ptr(stats, "stats", 8)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (int e = check_device()) return e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 rows(static_cast<unsigned>(B * N), static_cast<unsigned>(heads), static_cast<unsigned>((N + kQ - 1) / kQ));
  GTK_ATTN_LAUNCH(dq_kernel, rows);
  if (int e = check_launch("attention core backward (dq)")) return e;
  GTK_ATTN_LAUNCH(dkv_kernel, rows);
  if (int e = check_launch("attention core backward (dk, dv)")) return e;
  const dim3 bias(static_cast<unsigned>(B * heads), static_cast<unsigned>((N + kQ - 1) / kQ),
                  static_cast<unsigned>((N + kT - 1) / kT));
  GTK_ATTN_LAUNCH(dtri_kernel, bias);
  return check_launch("attention core backward (dtri)");
}

}  // extern "C"
