// General-shape path of the triangle blocks and the pair transition (see general.h).
//
// Data flow (fp32 unless noted; P = B*N*N pairs in the block's own frame, which is z^T for
// the ending-node attention):
//   TriMul     zn[P][c_z] = LN_in(z)
//              Y[P][4c + c_z] = zn (W_ap | W_ag | W_bp | W_bg | W_g)^T + b
//              a, b fp16 planes [B][N][c][ld] = proj * sigmoid(gate) * mask, pair-transposed
//              x planes = K2 contraction (the tcgen05 kernel of trimul.cu), stored times 1/N
//              xn[P][c] = LN_out(x)                      (in zn's buffer)
//              out = z + sigmoid(Y_g) * (xn W_z^T + b_z)
//              (reference src/genie_tk/triangle_mul.py:103-132)
//   TriAtt     zn[P][c_in] = LN(z or z^T)
//              Y[P][4hd + H] = zn (W_q | W_k | W_v | W_g | W_b)^T + (0 | 0 | 0 | b_g | 0)
//              q, k, v fp16 planes [B*N][H][N][Dp] and the triangle bias fp16 [B][H][N][Np]
//              o[P][hd] = softmax_k(q.k / sqrt(d) + inf (m - 1) + tri) v on the tensor-core
//              attention core of attn_bwd.cu (mma.sync, fp32 softmax)
//              out = z + (o * sigmoid(g)) W_o^T + b_o (the gate applied as the GEMM loads o),
//              rows written back in z's frame
//              (reference triangle_attention.py:100-143, primitives.py:114-178)
//   Transition zn = LN(z); h[P][n c] = relu(zn W_1^T + b_1); out = (z + h W_2^T + b_2) * m
//              (reference pair_transform.py:64-84, :190-193)
// LayerNorms, projections and the transition are fp32 arithmetic on the CUDA cores; the
// contraction and the attention core run on tensor cores with fp16 operands (a clamp to the
// fp16 range is reported in the status word). LayerNorm and the softmax use the reference's
// eps (1e-5) and additive mask value.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "attn_core.h"
#include "general.h"

namespace gtk {
namespace gen {

constexpr float kLog2eF = 1.4426950408889634f;

// Memory row of pair p = (b, r, c) of a block's frame: p itself, or (b, c, r) in the z^T frame.
__device__ __forceinline__ int64_t frame_row(int64_t p, int64_t N, int tr) {
  if (!tr) return p;
  const int64_t NN = N * N;
  const int64_t b = p / NN, rem = p - b * NN, r = rem / N, c = rem - r * N;
  return b * NN + c * N + r;
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------------------
// LayerNorm of pair rows, one warp per row: out[p] = LN(x[frame_row(p)]) * gamma + beta.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    ln_kernel(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
              float* __restrict__ out, int64_t rows, int D, int64_t N, int tr, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const float inv = 1.f / static_cast<float>(D);
  for (int64_t p = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < rows; p += nw) {
    const float* xr = x + frame_row(p, N, tr) * D;
    float s = 0.f;
    for (int c = lane; c < D; c += 32) s += xr[c];
    const float mean = warp_sum(s) * inv;
    float v = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float d = xr[c] - mean;
      v = fmaf(d, d, v);
    }
    const float rstd = rsqrtf(warp_sum(v) * inv + eps);
    float* o = out + p * D;
    for (int c = lane; c < D; c += 32) o[c] = fmaf((xr[c] - mean) * rstd, gamma[c], beta[c]);
  }
}

// ---------------------------------------------------------------------------------------
// C = A W^T (+ epilogue): A [M][K] (pitch lda), W [n_out][K] (pitch ldw), fp32 in memory.
// Tensor cores: mma.sync m16n8k8 with TF32 operands and fp32 accumulation. kSplit = 1 rounds
// each operand to TF32 (10-bit mantissa, the precision class of the tuned kernels' fp16
// operands); kSplit = 3 splits each operand into a TF32 head and a TF32 tail, x = hi + lo,
// and accumulates hi*hi + hi*lo + lo*hi (3xTF32: products to ~2^-22, fp32-level results).
// CTA tile 128 x 128 (8 warps of 32 x 64), K in steps of 32 through shared memory (double
// buffered; the next step's global loads -- 16-byte vectors when the pitches allow -- are in
// flight while this one multiplies).
// ---------------------------------------------------------------------------------------
enum EpiMode : int { kStore = 0, kRelu = 1, kGateRes = 2, kRes = 3, kResMask = 4 };

struct Epi {
  int mode;
  const float* bias;  // [n_out] or nullptr
  float* out;         // kStore / kRelu: [M][ldo]; else pair rows (frame_row), ldo = channels
  int64_t ldo;
  const float* z;     // residual pair tensor (may equal out; nullptr: no residual)
  int64_t N;          // pairs per side, for the pair-row mapping and the dropout vector
  int tr;             // rows of `out` / `z` are in the z^T frame
  const float* gate;  // kGateRes: gate logits [M][ldg]
  int64_t ldg;
  const float* mask;  // kResMask: [M] (nullptr: ones)
  DropArgs drop;      // kGateRes / kRes: channel dropout (keep == nullptr: none)
};

constexpr int kBM = 128, kBN = 128, kBK = 32;
constexpr int kBP = kBK + 4;  // shared pitch (floats): conflict-free fragment loads
constexpr int kGemmSmem = 2 * (kBM + kBN) * kBP * 4;  // two stages of the A and W tiles

// What the GEMM applies to A's elements as it loads them: nothing, a LayerNorm of each row
// (the CTA computes its rows' mean and 1/std first), a sigmoid gate, or fp16 A.
enum ProMode : int { kProNone = 0, kProLn = 1, kProGate = 2, kProHalf = 3 };

struct Pro {
  const float* gamma;  // kProLn
  const float* beta;
  float eps;
  const float* gate;   // kProGate: [M][ldg]
  int64_t ldg;
  const __half* ah;    // kProHalf: A is fp16 (this pointer, pitch lda) instead of fp32
};

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int kPro, int kSplit>
__global__ void __launch_bounds__(256, kSplit == 1 ? 2 : 1)
    gemm_kernel(const float* __restrict__ A, int64_t M, int K, int64_t lda, const float* __restrict__ W, int n_out,
                int64_t ldw, const Epi e, const Pro pro, int n_tiles_n, int vec) {
  extern __shared__ __align__(16) float gsm[];
  float (*As)[kBM][kBP] = reinterpret_cast<float (*)[kBM][kBP]>(gsm);
  float (*Ws)[kBN][kBP] = reinterpret_cast<float (*)[kBN][kBP]>(gsm + 2 * kBM * kBP);
  __shared__ float mean_s[kPro == kProLn ? kBM : 1], rstd_s[kPro == kProLn ? kBM : 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp & 3, wn = warp >> 2, g = lane >> 2, t = lane & 3;
  const int64_t tile = blockIdx.x;
  const int nt_idx = static_cast<int>(tile % n_tiles_n);  // the N tiles of one M block run side by side
  const int64_t m0 = (tile / n_tiles_n) * kBM;
  const int n0 = nt_idx * kBN;
  if constexpr (kPro == kProLn) {
    const float inv = 1.f / static_cast<float>(K);
    for (int r = warp; r < kBM; r += 8) {
      const int64_t m = m0 + r;
      float mean = 0.f, rstd = 0.f;
      if (m < M) {
        const float* xr = A + m * lda;
        float sum = 0.f;
        for (int k = lane; k < K; k += 32) sum += xr[k];
        mean = warp_sum(sum) * inv;
        float var = 0.f;
        for (int k = lane; k < K; k += 32) {
          const float dx = xr[k] - mean;
          var = fmaf(dx, dx, var);
        }
        rstd = rsqrtf(warp_sum(var) * inv + pro.eps);
      }
      if (lane == 0) {
        mean_s[r] = mean;
        rstd_s[r] = rstd;
      }
    }
    __syncthreads();
  }
  // global -> registers. Thread: rows (tid >> 3) + 32 u, columns 4 (tid & 7) .. +3 of the
  // 32-column step (16-byte vectors when `vec`: pitches and bases 16-byte aligned, K % 4 == 0).
  float ra[4][4], rw[4][4];
  const int lr = tid >> 3, lc = (tid & 7) * 4;
  auto xform = [&](float x, int64_t m, int r, int k) {
    if constexpr (kPro == kProLn) x = fmaf((x - mean_s[r]) * rstd_s[r], pro.gamma[k], pro.beta[k]);
    if constexpr (kPro == kProGate) x *= sigmoid_f(pro.gate[m * pro.ldg + k]);
    return x;
  };
  auto load = [&](int k0) {
    const int k = k0 + lc;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = lr + 32 * u;
      const int64_t m = m0 + r;
      const int n = n0 + r;
      float x[4] = {0.f, 0.f, 0.f, 0.f}, y[4] = {0.f, 0.f, 0.f, 0.f};
      if (m < M) {
        if (vec && k < K) {
          if constexpr (kPro == kProHalf) {
            const uint2 h = *reinterpret_cast<const uint2*>(pro.ah + m * lda + k);
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
            x[0] = f0.x, x[1] = f0.y, x[2] = f1.x, x[3] = f1.y;
          } else {
            const float4 f = *reinterpret_cast<const float4*>(A + m * lda + k);
            x[0] = f.x, x[1] = f.y, x[2] = f.z, x[3] = f.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (k + q < K) {
              if constexpr (kPro == kProHalf)
                x[q] = __half2float(pro.ah[m * lda + k + q]);
              else
                x[q] = A[m * lda + k + q];
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) x[q] = k + q < K ? xform(x[q], m, r, k + q) : 0.f;
      }
      if (n < n_out) {
        if (vec && k < K) {
          const float4 f = *reinterpret_cast<const float4*>(W + static_cast<int64_t>(n) * ldw + k);
          y[0] = f.x, y[1] = f.y, y[2] = f.z, y[3] = f.w;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (k + q < K) y[q] = W[static_cast<int64_t>(n) * ldw + k + q];
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        ra[u][q] = x[q];
        rw[u][q] = y[q];
      }
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = lr + 32 * u;
      *reinterpret_cast<float4*>(&As[buf][r][lc]) = make_float4(ra[u][0], ra[u][1], ra[u][2], ra[u][3]);
      *reinterpret_cast<float4*>(&Ws[buf][r][lc]) = make_float4(rw[u][0], rw[u][1], rw[u][2], rw[u][3]);
    }
  };
  float acc[2][8][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[a][b][0] = acc[a][b][1] = acc[a][b][2] = acc[a][b][3] = 0.f;
  load(0);
  store(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += kBK, buf ^= 1) {
    const bool more = k0 + kBK < K;
    if (more) load(k0 + kBK);
#pragma unroll
    for (int k8 = 0; k8 < kBK; k8 += 8) {
      uint32_t ah[2][4], al[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int r = wm * 32 + mt * 16 + g;
        const float x[4] = {As[buf][r][k8 + t], As[buf][r + 8][k8 + t], As[buf][r][k8 + t + 4],
                            As[buf][r + 8][k8 + t + 4]};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          ah[mt][q] = tf32_rna(x[q]);
          if constexpr (kSplit == 3) al[mt][q] = tf32_rna(x[q] - __uint_as_float(ah[mt][q]));
        }
      }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int c = wn * 64 + nt * 8 + g;
        const float y0 = Ws[buf][c][k8 + t], y1 = Ws[buf][c][k8 + t + 4];
        const uint32_t bh0 = tf32_rna(y0), bh1 = tf32_rna(y1);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          if constexpr (kSplit == 3) {
            const uint32_t bl0 = tf32_rna(y0 - __uint_as_float(bh0)), bl1 = tf32_rna(y1 - __uint_as_float(bh1));
            mma_tf32(acc[mt][nt], al[mt], bh0, bh1);
            mma_tf32(acc[mt][nt], ah[mt], bl0, bl1);
          }
          mma_tf32(acc[mt][nt], ah[mt], bh0, bh1);
        }
      }
    }
    if (more) store(buf ^ 1);  // buf ^ 1 was last read before the previous barrier
    __syncthreads();
  }
  // the tile through shared memory (the operand stages are free now), then row by row: a warp
  // owns 16 rows, a lane 4 consecutive columns, so each row leaves as 512 contiguous bytes
  float (*Cs)[kBN + 4] = reinterpret_cast<float (*)[kBN + 4]>(gsm);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        *reinterpret_cast<float2*>(&Cs[wm * 32 + mt * 16 + g + h * 8][wn * 64 + nt * 8 + 2 * t]) =
            make_float2(acc[mt][nt][2 * h], acc[mt][nt][2 * h + 1]);
  __syncthreads();
  const int c0 = lane * 4, n = n0 + c0;
  if (n >= n_out) return;
  const bool full = n + 3 < n_out;
  float bv[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) bv[q] = (e.bias && n + q < n_out) ? e.bias[n + q] : 0.f;
  const bool vec_out = full && (e.ldo % 4 == 0) && !(reinterpret_cast<uintptr_t>(e.out) & 15);
  for (int rr = 0; rr < 16; ++rr) {
    const int r = warp * 16 + rr;
    const int64_t m = m0 + r;
    if (m >= M) break;
    const float4 cv = *reinterpret_cast<const float4*>(&Cs[r][c0]);
    float v[4] = {cv.x + bv[0], cv.y + bv[1], cv.z + bv[2], cv.w + bv[3]};
    int64_t row = m;
    float mul = 1.f;
    const float* zr = nullptr;
    if (e.mode == kRelu) {
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = fmaxf(v[q], 0.f);
    } else if (e.mode == kResMask) {
      zr = e.z;
      mul = e.mask ? e.mask[m] : 1.f;
    } else if (e.mode == kGateRes || e.mode == kRes) {
      row = frame_row(m, e.N, e.tr);
      zr = e.z;
      if (e.mode == kGateRes)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (n + q < n_out) v[q] *= sigmoid_f(e.gate[m * e.ldg + n + q]);
      if (e.drop.keep != nullptr) {
        const int64_t NN = e.N * e.N;
        const int64_t b = m / NN, rem = m - b * NN, ri = rem / e.N, j = rem - ri * e.N;
        // n .. n+3 lie in one 128-channel group of the keep vector
        const uint4 keep = __ldg(e.drop.keep + (b * e.drop.ld + (e.drop.by_row ? ri : j)) * e.drop.groups + (n >> 7));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int nq = n + q;
          v[q] *= ((drop_word(keep, (nq & 127) >> 5) >> (nq & 31)) & 1u) ? e.drop.scale : 0.f;
        }
      }
    }
    float* o = e.out + row * e.ldo + n;
    if (vec_out) {
      if (zr) {
        const float4 zv = *reinterpret_cast<const float4*>(zr + row * e.ldo + n);
        v[0] += zv.x, v[1] += zv.y, v[2] += zv.z, v[3] += zv.w;
      }
      *reinterpret_cast<float4*>(o) = make_float4(v[0] * mul, v[1] * mul, v[2] * mul, v[3] * mul);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (n + q < n_out) o[q] = ((zr ? zr[row * e.ldo + n + q] : 0.f) + v[q]) * mul;
    }
  }
}

// ---------------------------------------------------------------------------------------
// TriMul a, b planes: plane element ((b*N + i)*c + ch)*ld + k = a[b, i, k, ch] with
// a = Y[p][ch] * sigmoid(Y[p][c + ch]) * m[p], p = (b*N + i)*N + k (b from columns 2c, 3c);
// zero for k >= N. 32 x 32 tiles transposed through shared memory.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    trimul_planes_kernel(const float* __restrict__ Y, int64_t ldy, const float* __restrict__ mask,
                         __half* __restrict__ a, __half* __restrict__ b, int64_t N, int c, int64_t ld,
                         uint32_t* status) {
  __shared__ float ta[32][33], tb[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;  // b*N + i
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int c0 = blockIdx.z * 32;
  for (int kk = ty; kk < 32; kk += 8) {
    const int64_t k = k0 + kk;
    const int ch = c0 + tx;
    float va = 0.f, vb = 0.f;
    if (k < N && ch < c) {
      const int64_t p = row * N + k;
      const float* y = Y + p * ldy;
      const float m = mask ? mask[p] : 1.f;
      va = y[ch] * sigmoid_f(y[c + ch]) * m;
      vb = y[2 * c + ch] * sigmoid_f(y[3 * c + ch]) * m;
    }
    ta[kk][tx] = va;
    tb[kk][tx] = vb;
  }
  __syncthreads();
  uint32_t sat = 0;  // an a / b value beyond the fp16 range was clamped
  for (int cc = ty; cc < 32; cc += 8) {
    const int ch = c0 + cc;
    const int64_t k = k0 + tx;
    if (ch < c && k < ld) {
      const int64_t o = (row * c + ch) * ld + k;
      a[o] = f16_sat_chk(ta[tx][cc], sat);
      b[o] = f16_sat_chk(tb[tx][cc], sat);
    }
  }
  flag_saturation(sat, status);
}

// ---------------------------------------------------------------------------------------
// LN_out of the contraction: xn[p][ch] = LN over ch of x[b][i][ch][j] * gamma + beta, with
// p = (b*N + i)*N + j. x is stored times 1/N; LayerNorm is scale-invariant once eps is
// scaled by the same factor squared, which the caller does.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    x_ln_kernel(const __half* __restrict__ x, int64_t ld, int64_t N, int c, const float* __restrict__ gamma,
                const float* __restrict__ beta, float eps, float* __restrict__ xn) {
  extern __shared__ float xs[];  // [c][33]
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * 32;
  for (int ch = ty; ch < c; ch += 8) {
    const int64_t j = j0 + tx;
    xs[ch * 33 + tx] = j < N ? __half2float(x[(row * c + ch) * ld + j]) : 0.f;
  }
  __syncthreads();
  const float inv = 1.f / static_cast<float>(c);
  for (int jj = ty; jj < 32; jj += 8) {
    const int64_t j = j0 + jj;
    if (j >= N) break;  // uniform across the warp
    float s = 0.f;
    for (int ch = tx; ch < c; ch += 32) s += xs[ch * 33 + jj];
    const float mean = warp_sum(s) * inv;
    float v = 0.f;
    for (int ch = tx; ch < c; ch += 32) {
      const float d = xs[ch * 33 + jj] - mean;
      v = fmaf(d, d, v);
    }
    const float rstd = rsqrtf(warp_sum(v) * inv + eps);
    float* o = xn + (row * N + j) * c;
    for (int ch = tx; ch < c; ch += 32) o[ch] = fmaf((xs[ch * 33 + jj] - mean) * rstd, gamma[ch], beta[ch]);
  }
}

// ---------------------------------------------------------------------------------------
// Triangle bias as the attention core's fp16 plane: trih[b][h][j][k] = Y[(b*N + j)*N + k][col0 + h]
// for k < N, zero for N <= k < Np. Eight keys per thread.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    tri_bias_f16_kernel(const float* __restrict__ Y, int64_t ldy, int col0, int H, int64_t B, int64_t N, int64_t Np,
                        __half* __restrict__ trih) {
  const int64_t C = Np / 8;
  const int64_t total = B * H * N * C;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t % C;
    int64_t r = t / C;
    const int64_t j = r % N;
    r /= N;
    const int64_t h = r % H, b = r / H;
    __align__(16) __half v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t k = c * 8 + u;
      v[u] = __float2half_rn(k < N ? Y[((b * N + j) * N + k) * ldy + col0 + h] : 0.f);
    }
    *reinterpret_cast<uint4*>(trih + t * 8) = *reinterpret_cast<const uint4*>(v);
  }
}

// ---------------------------------------------------------------------------------------
// Operands of the tuned attention core (triatt.cu, 4 heads of 32) for a general block with
// 4 heads of d <= 32, zero-padded to 32:
//   gate[p][h*32 + e] = sigmoid(Y[p][3hd + h*d + e]) (0 for e >= d), fp16 [P][128];
//   bias[(j*B*4 + b*4 + h)*ldn + k] = Y[(b*N + j)*N + k][4hd + h] * log2 e, bf16, 0 for k >= N;
//   wpad[o][h*32 + e] = W_o[o][h*d + e] (0 for e >= d), so og [P][128] multiplies it directly.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    k4_gate_kernel(const float* __restrict__ Y, int64_t ldy, int col0, int d, int64_t P, __half* __restrict__ gate) {
  const int64_t total = P * 16;  // 16 chunks of 8 channels per pair
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = t >> 4;
    const int c = static_cast<int>(t & 15), h = c >> 2, e0 = (c & 3) * 8;
    const float* y = Y + p * ldy + col0 + h * d;
    __align__(16) __half v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __float2half_rn(e0 + u < d ? sigmoid_f(y[e0 + u]) : 0.f);
    *reinterpret_cast<uint4*>(gate + t * 8) = *reinterpret_cast<const uint4*>(v);
  }
}

__global__ void __launch_bounds__(256)
    k4_bias_kernel(const float* __restrict__ Y, int64_t ldy, int col0, int64_t B, int64_t N, int64_t ldn,
                   __nv_bfloat16* __restrict__ bias) {
  const int64_t C = ldn / 8;
  const int64_t total = N * B * 4 * C;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = t % C;
    int64_t r = t / C;  // r = j * B * 4 + b * 4 + h
    const int h = static_cast<int>(r & 3);
    r >>= 2;
    const int64_t b = r % B, j = r / B;
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t k = c * 8 + u;
      v[u] = __float2bfloat16_rn(k < N ? Y[((b * N + j) * N + k) * ldy + col0 + h] * 1.4426950408889634f : 0.f);
    }
    *reinterpret_cast<uint4*>(bias + t * 8) = *reinterpret_cast<const uint4*>(v);
  }
}

__global__ void __launch_bounds__(128)
    wo_pad_kernel(const float* __restrict__ wo, int cin, int d, float* __restrict__ wpad) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < cin * 128; t += gridDim.x * blockDim.x) {
    const int o = t >> 7, c = t & 127, h = c >> 5, e = c & 31;
    wpad[t] = e < d ? wo[static_cast<int64_t>(o) * 4 * d + h * d + e] : 0.f;
  }
}

// ---------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------
static size_t a256(size_t x) { return (x + 255) / 256 * 256; }

static int grid_rows(int64_t rows, int per_block) {
  const int64_t need = (rows + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  return static_cast<int>(need < 1 ? 1 : (need < cap ? need : cap));
}

static int launch_ln(const float* x, const float* gamma, const float* beta, float* out, int64_t rows, int D, int64_t N,
                     int tr, cudaStream_t st) {
  ln_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(x, gamma, beta, out, rows, D, N, tr, 1e-5f);
  return check_launch("general ln_kernel");
}

// The general blocks' GEMMs (TF32 operands) and the fp32-accurate form (3xTF32) of
// gtk_linear / gtk_layernorm_linear, with any prologue.
template <int kPro, int kSplit>
static int launch_gemm_t(const float* A, int64_t M, int K, int64_t lda, const float* W, int n_out, int64_t ldw,
                         const Epi& e, const Pro& pro, cudaStream_t st, const char* what) {
  const int64_t mt = (M + kBM - 1) / kBM, ntn = (n_out + kBN - 1) / kBN;
  if (mt * ntn > 2147483647) return fail(GTK_ERR_INVALID_ARG, std::string(what) + ": too many rows");
  const void* abase = kPro == kProHalf ? static_cast<const void*>(pro.ah) : static_cast<const void*>(A);
  const uintptr_t amask = kPro == kProHalf ? 7 : 15;
  const int vec = (K % 4 == 0) && (lda % 4 == 0) && (ldw % 4 == 0) && !(reinterpret_cast<uintptr_t>(abase) & amask) &&
                  !(reinterpret_cast<uintptr_t>(W) & 15);
  const void* kern = reinterpret_cast<const void*>(gemm_kernel<kPro, kSplit>);
  if (int e2 = ensure_smem(kern, kGemmSmem)) return e2;
  gemm_kernel<kPro, kSplit><<<static_cast<unsigned>(mt * ntn), 256, kGemmSmem, st>>>(A, M, K, lda, W, n_out, ldw, e,
                                                                                  pro, static_cast<int>(ntn), vec);
  return check_launch(what);
}

static int launch_gemm(const float* A, int64_t M, int K, int64_t lda, const float* W, int n_out, int64_t ldw,
                       const Epi& e, cudaStream_t st) {
  return launch_gemm_t<kProNone, 1>(A, M, K, lda, W, n_out, ldw, e, Pro{}, st, "general gemm_kernel");
}

static Epi epi(int mode, const float* bias, float* out, int64_t ldo) {
  Epi e{};
  e.mode = mode;
  e.bias = bias;
  e.out = out;
  e.ldo = ldo;
  e.N = 1;
  return e;
}

static int copy_d2d(float* dst, const float* src, size_t n, cudaStream_t st) {
  if (!src) return cudaMemsetAsync(dst, 0, n * 4, st) == cudaSuccess ? GTK_OK : fail(GTK_ERR_CUDA, "memset failed");
  const cudaError_t e = cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, st);
  return e == cudaSuccess ? GTK_OK : fail(GTK_ERR_CUDA, std::string("packing copy failed: ") + cudaGetErrorString(e));
}

static int common_args(const float* z, const float* out, const void* packed, void* workspace, const float* mask,
                       int64_t B, int64_t N) {
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535)) return fail(GTK_ERR_INVALID_ARG, "bad B/N");
  if (int e = check_ptr(z, "z", 4)) return e;
  if (int e = check_ptr(out, "out", 4)) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  return GTK_OK;
}

static int drop_channels(const DropArgs& drop, int channels) {
  if (drop.keep && drop.groups * 128 < channels)
    return fail(GTK_ERR_INVALID_ARG, "dropout keep vectors hold " + std::to_string(drop.groups * 128) +
                                         " channels; this block has " + std::to_string(channels));
  return GTK_OK;
}

// ----------------------------- triangle multiplication ---------------------------------
// packed floats: W1 [(4c + c_z) x c_z] | b1 [4c + c_z] | W_z [c_z x c] | b_z [c_z] |
//                ln_in w, b [c_z] | ln_out w, b [c]
struct TmPack {
  size_t w1, b1, wz, bz, liw, lib, low, lob, floats;
};
static TmPack tm_pack(int cz, int c) {
  TmPack p{};
  const size_t rows = 4 * static_cast<size_t>(c) + cz;
  p.w1 = 0;
  p.b1 = p.w1 + rows * cz;
  p.wz = p.b1 + rows;
  p.bz = p.wz + static_cast<size_t>(cz) * c;
  p.liw = p.bz + cz;
  p.lib = p.liw + cz;
  p.low = p.lib + cz;
  p.lob = p.low + c;
  p.floats = p.lob + c;
  return p;
}

struct TmWs {
  size_t zn, y, a, b, x, total;
};
static TmWs tm_ws(int64_t B, int64_t N, int cz, int c) {
  TmWs w{};
  const size_t P = static_cast<size_t>(B) * N * N;
  const size_t plane = a256(static_cast<size_t>(B) * N * c * gtk_plane_pitch(N) * 2);
  w.zn = 0;
  w.y = a256(P * (cz > c ? cz : c) * 4);
  w.a = w.y + a256(P * (4 * static_cast<size_t>(c) + cz) * 4);
  w.b = w.a + plane;
  w.x = w.b + plane;
  w.total = w.x + plane;
  return w;
}

int trimul_check(int c_z, int c_hidden) {
  if (c_z < 1 || c_hidden < 1 || c_z > kMaxChannels || c_hidden > kMaxChannels)
    return fail(GTK_ERR_UNSUPPORTED, "trimul: c_z and c_hidden must be in 1.." + std::to_string(kMaxChannels));
  return GTK_OK;
}

size_t trimul_packed_bytes(int c_z, int c_hidden) {
  if (c_z < 1 || c_hidden < 1 || c_z > kMaxChannels || c_hidden > kMaxChannels) return 0;
  return a256(tm_pack(c_z, c_hidden).floats * 4);
}

int trimul_pack(const gtk_trimul_params* params, int c_z, int c_hidden, void* packed, size_t packed_bytes,
                void* stream) {
  if (int e = trimul_check(c_z, c_hidden)) return e;
  if (!params) return fail(GTK_ERR_INVALID_ARG, "params is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < trimul_packed_bytes(c_z, c_hidden)) return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  const float* const* pp = reinterpret_cast<const float* const*>(params);
  for (int i = 0; i < 16; ++i)
    if (!pp[i]) return fail(GTK_ERR_INVALID_ARG, "a trimul parameter pointer is NULL");
  if (int e = check_device()) return e;
  const TmPack L = tm_pack(c_z, c_hidden);
  float* f = static_cast<float*>(packed);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t c = c_hidden, cz = c_z;
  const gtk_trimul_params& p = *params;
  const float* w1_src[5] = {p.a_p_w, p.a_g_w, p.b_p_w, p.b_g_w, p.g_w};
  const float* b1_src[5] = {p.a_p_b, p.a_g_b, p.b_p_b, p.b_g_b, p.g_b};
  for (int k = 0; k < 5; ++k) {
    const size_t rows = k < 4 ? c : cz;
    if (int e = copy_d2d(f + L.w1 + k * c * cz, w1_src[k], rows * cz, st)) return e;
    if (int e = copy_d2d(f + L.b1 + k * c, b1_src[k], rows, st)) return e;
  }
  if (int e = copy_d2d(f + L.wz, p.z_w, cz * c, st)) return e;
  if (int e = copy_d2d(f + L.bz, p.z_b, cz, st)) return e;
  if (int e = copy_d2d(f + L.liw, p.ln_in_w, cz, st)) return e;
  if (int e = copy_d2d(f + L.lib, p.ln_in_b, cz, st)) return e;
  if (int e = copy_d2d(f + L.low, p.ln_out_w, c, st)) return e;
  return copy_d2d(f + L.lob, p.ln_out_b, c, st);
}

size_t trimul_workspace_bytes(int64_t B, int64_t N, int c_z, int c_hidden) {
  if (c_z < 1 || c_hidden < 1 || c_z > kMaxChannels || c_hidden > kMaxChannels || B < 1 || N < 1) return 0;
  return tm_ws(B, N, c_z, c_hidden).total;
}

int trimul_forward(int outgoing, const float* z, const float* mask, const void* packed, float* out, int add_residual,
                   const DropArgs& drop, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_z,
                   int c_hidden, uint32_t* status, void* stream) {
  if (int e = trimul_check(c_z, c_hidden)) return e;
  if (int e = common_args(z, out, packed, workspace, mask, B, N)) return e;
  if (int e = drop_channels(drop, c_z)) return e;
  const TmWs w = tm_ws(B, N, c_z, c_hidden);
  if (workspace_bytes < w.total) return fail(GTK_ERR_WORKSPACE, "trimul: workspace too small");
  if (int e = check_device()) return e;
  const TmPack L = tm_pack(c_z, c_hidden);
  const float* pk = static_cast<const float*>(packed);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* zn = reinterpret_cast<float*>(ws + w.zn);
  float* Y = reinterpret_cast<float*>(ws + w.y);
  __half* ap = reinterpret_cast<__half*>(ws + w.a);
  __half* bp = reinterpret_cast<__half*>(ws + w.b);
  __half* xp = reinterpret_cast<__half*>(ws + w.x);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t P = B * N * N;
  const int c = c_hidden;
  const int64_t ldy = 4 * static_cast<int64_t>(c) + c_z, ld = gtk_plane_pitch(N);
  if (int e = launch_ln(z, pk + L.liw, pk + L.lib, zn, P, c_z, N, 0, st)) return e;
  if (int e = launch_gemm(zn, P, c_z, c_z, pk + L.w1, static_cast<int>(ldy), c_z, epi(kStore, pk + L.b1, Y, ldy), st))
    return e;
  {
    const int64_t kb = (ld + 31) / 32;
    if (B * N > 2147483647 || kb > 65535) return fail(GTK_ERR_INVALID_ARG, "trimul: N too large");
    dim3 grid(static_cast<unsigned>(B * N), static_cast<unsigned>(kb), static_cast<unsigned>((c + 31) / 32));
    trimul_planes_kernel<<<grid, 256, 0, st>>>(Y, ldy, mask, ap, bp, N, c, ld, status);
    if (int e = check_launch("general trimul_planes_kernel")) return e;
  }
  const float xs = 1.f / static_cast<float>(N);
  if (int e = gtk_trimul_contract(outgoing, ap, bp, xp, B, c, N, N, N, ld, ld, ld, xs, status, stream)) return e;
  {
    // the kernel's dynamic shared memory limit is set once, to the largest channel count
    const int smem = c * 33 * 4;
    if (int e = ensure_smem(reinterpret_cast<const void*>(x_ln_kernel), kMaxChannels * 33 * 4)) return e;
    dim3 grid(static_cast<unsigned>(B * N), static_cast<unsigned>((N + 31) / 32));
    x_ln_kernel<<<grid, 256, smem, st>>>(xp, ld, N, c, pk + L.low, pk + L.lob, 1e-5f * xs * xs, zn);
    if (int e = check_launch("general x_ln_kernel")) return e;
  }
  Epi e = epi(kGateRes, pk + L.bz, out, c_z);
  e.z = add_residual ? z : nullptr;
  e.N = N;
  e.tr = 0;
  e.gate = Y + 4 * static_cast<int64_t>(c);
  e.ldg = ldy;
  e.drop = drop;
  return launch_gemm(zn, P, c, c, pk + L.wz, c_z, c, e, st);
}

// --------------------------------- triangle attention -----------------------------------
// packed floats: W [(4hd + H) x c_in] (q | k | v | g | bias) | b [4hd + H] (0 | 0 | 0 | b_g | 0) |
//                W_o [c_in x hd] | b_o [c_in] | ln w, b [c_in]
struct TaPack {
  size_t w, b, wo, bo, lw, lb, floats;
};
static TaPack ta_pack(int cin, int hd, int H) {
  TaPack p{};
  const size_t rows = 4 * static_cast<size_t>(hd) + H;
  p.w = 0;
  p.b = rows * cin;
  p.wo = p.b + rows;
  p.bo = p.wo + static_cast<size_t>(cin) * hd;
  p.lw = p.bo + cin;
  p.lb = p.lw + cin;
  p.floats = p.lb + cin;
  return p;
}

// The general attention's core runs on the tuned tcgen05 core (triatt.cu) when it has that
// core's 4 heads and head_dim <= 32 (zero-padded to 32; the reference's default 32 = 4 x 8
// among them), else on the mma.sync core of attn_bwd.cu.
static bool ta_tuned_core(int hd, int H) { return H == 4 && hd % 4 == 0 && hd / 4 <= 32; }

// zn (LayerNorm output) | Y (projections) | then either the tuned core's workspace
// (q, k, v, gate, og, bias) and the head-padded W_o, or the fp16 bias plane, o and the fp16
// q, k, v planes of the mma.sync core.
struct TaWs {
  size_t zn, y, tri, og, q, k, v, k4, wpad, total;
};
static TaWs ta_ws(int64_t B, int64_t N, int cin, int hd, int H) {
  TaWs w{};
  const size_t P = static_cast<size_t>(B) * N * N;
  w.zn = 0;
  w.y = a256(P * cin * 4);
  const size_t rest = w.y + a256(P * (4 * static_cast<size_t>(hd) + H) * 4);
  if (ta_tuned_core(hd, H)) {
    w.k4 = rest;
    w.wpad = w.k4 + a256(gtk_triatt_workspace_bytes(B, N, 128, 128, 4));
    w.total = w.wpad + a256(static_cast<size_t>(cin) * 128 * 4);
    return w;
  }
  const size_t plane = a256(P * H * attn::padded_head_dim(hd / H) * 2);
  w.tri = rest;
  w.og = w.tri + a256(static_cast<size_t>(B) * H * N * ((N + 7) / 8 * 8) * 2);
  w.q = w.og + a256(P * hd * 4);
  w.k = w.q + plane;
  w.v = w.k + plane;
  w.total = w.v + plane;
  return w;
}

int triatt_check(int c_in, int c_hidden, int heads) {
  if (c_in < 1 || c_in > kMaxChannels || heads < 1 || heads > kMaxHeads || c_hidden < heads ||
      c_hidden > kMaxChannels || c_hidden % heads != 0 || c_hidden / heads > kMaxHeadDim)
    return fail(GTK_ERR_UNSUPPORTED, "triatt: need c_in <= " + std::to_string(kMaxChannels) + ", 1 <= heads <= " +
                                         std::to_string(kMaxHeads) + ", c_hidden a multiple of heads with head_dim <= " +
                                         std::to_string(kMaxHeadDim));
  return GTK_OK;
}

size_t triatt_packed_bytes(int c_in, int c_hidden, int heads) {
  if (c_in < 1 || c_in > kMaxChannels || heads < 1 || heads > kMaxHeads || c_hidden < heads ||
      c_hidden > kMaxChannels || c_hidden % heads != 0 || c_hidden / heads > kMaxHeadDim)
    return 0;
  return a256(ta_pack(c_in, c_hidden, heads).floats * 4);
}

int triatt_pack(const gtk_triatt_params* params, int c_in, int c_hidden, int heads, void* packed,
                size_t packed_bytes, void* stream) {
  if (int e = triatt_check(c_in, c_hidden, heads)) return e;
  if (!params) return fail(GTK_ERR_INVALID_ARG, "params is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < triatt_packed_bytes(c_in, c_hidden, heads))
    return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  const float* const* pp = reinterpret_cast<const float* const*>(params);
  for (int i = 0; i < 10; ++i)
    if (!pp[i]) return fail(GTK_ERR_INVALID_ARG, "a triatt parameter pointer is NULL");
  if (int e = check_device()) return e;
  const TaPack L = ta_pack(c_in, c_hidden, heads);
  float* f = static_cast<float*>(packed);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t hd = c_hidden, cin = c_in;
  const gtk_triatt_params& p = *params;
  const float* w_src[4] = {p.q_w, p.k_w, p.v_w, p.g_w};
  for (int k = 0; k < 4; ++k)
    if (int e = copy_d2d(f + L.w + k * hd * cin, w_src[k], hd * cin, st)) return e;
  if (int e = copy_d2d(f + L.w + 4 * hd * cin, p.bias_w, static_cast<size_t>(heads) * cin, st)) return e;
  if (int e = copy_d2d(f + L.b, nullptr, 3 * hd, st)) return e;
  if (int e = copy_d2d(f + L.b + 3 * hd, p.g_b, hd, st)) return e;
  if (int e = copy_d2d(f + L.b + 4 * hd, nullptr, heads, st)) return e;
  if (int e = copy_d2d(f + L.wo, p.o_w, cin * hd, st)) return e;
  if (int e = copy_d2d(f + L.bo, p.o_b, cin, st)) return e;
  if (int e = copy_d2d(f + L.lw, p.ln_w, cin, st)) return e;
  return copy_d2d(f + L.lb, p.ln_b, cin, st);
}

size_t triatt_workspace_bytes(int64_t B, int64_t N, int c_in, int c_hidden, int heads) {
  if (triatt_packed_bytes(c_in, c_hidden, heads) == 0 || B < 1 || N < 1) return 0;
  return ta_ws(B, N, c_in, c_hidden, heads).total;
}


int triatt_forward(int starting, const float* z, const float* mask, const void* packed, float* out,
                   int add_residual, const DropArgs& drop, void* workspace, size_t workspace_bytes, int64_t B,
                   int64_t N, int c_in, int c_hidden, int heads, float inf, uint32_t* status, void* stream) {
  if (int e = triatt_check(c_in, c_hidden, heads)) return e;
  if (int e = common_args(z, out, packed, workspace, mask, B, N)) return e;
  if (int e = drop_channels(drop, c_in)) return e;
  if (!std::isfinite(inf)) return fail(GTK_ERR_INVALID_ARG, "triatt: inf must be finite");
  const TaWs w = ta_ws(B, N, c_in, c_hidden, heads);
  if (workspace_bytes < w.total) return fail(GTK_ERR_WORKSPACE, "triatt: workspace too small");
  if (int e = check_device()) return e;
  const TaPack L = ta_pack(c_in, c_hidden, heads);
  const float* pk = static_cast<const float*>(packed);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* zn = reinterpret_cast<float*>(ws + w.zn);
  float* Y = reinterpret_cast<float*>(ws + w.y);
  float* og = reinterpret_cast<float*>(ws + w.og);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t P = B * N * N;
  const int hd = c_hidden, H = heads, d = c_hidden / heads;
  const int tr = starting ? 0 : 1;
  const int64_t ldy = 4 * static_cast<int64_t>(hd) + H;
  if (int e = launch_ln(z, pk + L.lw, pk + L.lb, zn, P, c_in, N, tr, st)) return e;
  if (int e = launch_gemm(zn, P, c_in, c_in, pk + L.w, static_cast<int>(ldy), c_in, epi(kStore, pk + L.b, Y, ldy),
                          st))
    return e;
  if (ta_tuned_core(hd, H)) {
    // the tuned tcgen05 core: q (times log2 e / sqrt(d)), k, v as its [B*N][4][N][32]
    // fp16 planes, the sigmoid gate and the bf16 log2 bias in its layouts
    int64_t off[7];
    if (int e = gtk_triatt_workspace_offsets(B, N, N, off)) return e;
    uint8_t* w4 = ws + w.k4;
    const float qs = kLog2eF / std::sqrt(static_cast<float>(d));
    if (int e = attn::launch_pack(Y, ldy, B, N, H, d, qs, reinterpret_cast<__half*>(w4 + off[0]), status, st, 32))
      return e;
    if (int e = attn::launch_pack(Y + hd, ldy, B, N, H, d, 1.f, reinterpret_cast<__half*>(w4 + off[1]), status, st,
                                  32))
      return e;
    if (int e = attn::launch_pack(Y + 2 * hd, ldy, B, N, H, d, 1.f, reinterpret_cast<__half*>(w4 + off[2]), status,
                                  st, 32))
      return e;
    k4_gate_kernel<<<grid_rows(P * 16, 256), 256, 0, st>>>(Y, ldy, 3 * hd, d, P,
                                                          reinterpret_cast<__half*>(w4 + off[3]));
    if (int e = check_launch("general k4_gate_kernel")) return e;
    const int64_t ldn = (N + 7) / 8 * 8;
    k4_bias_kernel<<<grid_rows(N * B * 4 * (ldn / 8), 256), 256, 0, st>>>(
        Y, ldy, 4 * hd, B, N, ldn, reinterpret_cast<__nv_bfloat16*>(w4 + off[5]));
    if (int e = check_launch("general k4_bias_kernel")) return e;
    if (int e = gtk_triatt_core(starting, mask, w4, B, N, N, 0, inf, status, stream)) return e;
    float* wpad = reinterpret_cast<float*>(ws + w.wpad);
    wo_pad_kernel<<<(c_in * 128 + 127) / 128, 128, 0, st>>>(pk + L.wo, c_in, d, wpad);
    if (int e = check_launch("general wo_pad_kernel")) return e;
    // out = z + og W_pad^T + b_o; og already carries the gate
    Epi e = epi(kRes, pk + L.bo, out, c_in);
    e.z = add_residual ? z : nullptr;
    e.N = N;
    e.tr = tr;
    e.drop = drop;
    Pro pro{};
    pro.ah = reinterpret_cast<const __half*>(w4 + off[4]);
      return launch_gemm_t<kProHalf, 1>(nullptr, P, 128, 128, wpad, c_in, 128, e, pro, st,
                                      "general gemm_kernel (tuned-core output)");
  }
  // the attention core on the tensor cores: q, k, v and the bias as fp16 planes
  __half* qh = reinterpret_cast<__half*>(ws + w.q);
  __half* kh = reinterpret_cast<__half*>(ws + w.k);
  __half* vh = reinterpret_cast<__half*>(ws + w.v);
  __half* trih = reinterpret_cast<__half*>(ws + w.tri);
  if (int e = attn::launch_pack(Y, ldy, B, N, H, d, 1.f, qh, status, st)) return e;
  if (int e = attn::launch_pack(Y + hd, ldy, B, N, H, d, 1.f, kh, status, st)) return e;
  if (int e = attn::launch_pack(Y + 2 * hd, ldy, B, N, H, d, 1.f, vh, status, st)) return e;
  {
    const int64_t Np = (N + 7) / 8 * 8;
    tri_bias_f16_kernel<<<grid_rows(B * H * N * (Np / 8), 256), 256, 0, st>>>(Y, ldy, 4 * hd, H, B, N, Np, trih);
    if (int e = check_launch("general tri_bias_f16_kernel")) return e;
  }
  // the mask in the block's frame: m[b, i, k] (starting) or m[b, k, i] (ending)
  if (int e = attn::launch_forward(qh, kh, vh, trih, mask, starting ? N : 1, starting ? 1 : N, B, N, H, d, inf, og,
                                   st))
    return e;
  // out = z + (o * sigmoid(g)) W_o^T + b_o, the gate applied as the GEMM loads o
  Epi e = epi(kRes, pk + L.bo, out, c_in);
  e.z = add_residual ? z : nullptr;
  e.N = N;
  e.tr = tr;
  e.drop = drop;
  Pro pro{};
  pro.gate = Y + 3 * hd;
  pro.ldg = ldy;
  return launch_gemm_t<kProGate, 1>(og, P, hd, hd, pk + L.wo, c_in, hd, e, pro, st,
                                    "general gemm_kernel (gated output)");
}

// ----------------------------------- pair transition -----------------------------------
// packed floats: W1 [nc x c] | b1 [nc] | W2 [c x nc] | b2 [c] | ln w, b [c]
struct TnPack {
  size_t w1, b1, w2, b2, lw, lb, floats;
};
static TnPack tn_pack(int c, int n) {
  TnPack p{};
  const size_t h = static_cast<size_t>(c) * n;
  p.w1 = 0;
  p.b1 = h * c;
  p.w2 = p.b1 + h;
  p.b2 = p.w2 + h * c;
  p.lw = p.b2 + c;
  p.lb = p.lw + c;
  p.floats = p.lb + c;
  return p;
}

int transition_check(int c_p, int n) {
  if (c_p < 1 || c_p > kMaxChannels || n < 1 || static_cast<int64_t>(c_p) * n > 4 * kMaxChannels)
    return fail(GTK_ERR_UNSUPPORTED, "transition: need 1 <= c_p <= " + std::to_string(kMaxChannels) +
                                         " and c_p * n <= " + std::to_string(4 * kMaxChannels));
  return GTK_OK;
}

size_t transition_packed_bytes(int c_p, int n) {
  if (c_p < 1 || c_p > kMaxChannels || n < 1 || static_cast<int64_t>(c_p) * n > 4 * kMaxChannels) return 0;
  return a256(tn_pack(c_p, n).floats * 4);
}

int transition_pack(const gtk_transition_params* params, int c_p, int n, void* packed, size_t packed_bytes,
                    void* stream) {
  if (int e = transition_check(c_p, n)) return e;
  if (!params || !params->ln_w || !params->ln_b || !params->w1 || !params->w2)
    return fail(GTK_ERR_INVALID_ARG, "transition_pack: a required parameter pointer is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < transition_packed_bytes(c_p, n)) return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  if (int e = check_device()) return e;
  const TnPack L = tn_pack(c_p, n);
  float* f = static_cast<float*>(packed);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t c = c_p, h = static_cast<size_t>(c_p) * n;
  if (int e = copy_d2d(f + L.w1, params->w1, h * c, st)) return e;
  if (int e = copy_d2d(f + L.b1, params->b1, h, st)) return e;
  if (int e = copy_d2d(f + L.w2, params->w2, c * h, st)) return e;
  if (int e = copy_d2d(f + L.b2, params->b2, c, st)) return e;
  if (int e = copy_d2d(f + L.lw, params->ln_w, c, st)) return e;
  return copy_d2d(f + L.lb, params->ln_b, c, st);
}

size_t transition_workspace_bytes(int64_t B, int64_t N, int c_p, int n) {
  if (transition_packed_bytes(c_p, n) == 0 || B < 1 || N < 1) return 0;
  const size_t P = static_cast<size_t>(B) * N * N;
  return a256(P * c_p * 4) + a256(P * static_cast<size_t>(c_p) * n * 4);
}

int transition_forward(const float* z, const float* mask, const void* packed, float* out, int add_residual,
                       void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_p, int n,
                       uint32_t* status, void* stream) {
  (void)status;
  if (int e = transition_check(c_p, n)) return e;
  if (int e = common_args(z, out, packed, workspace, mask, B, N)) return e;
  if (workspace_bytes < transition_workspace_bytes(B, N, c_p, n))
    return fail(GTK_ERR_WORKSPACE, "transition: workspace too small");
  if (int e = check_device()) return e;
  const TnPack L = tn_pack(c_p, n);
  const float* pk = static_cast<const float*>(packed);
  const size_t P = static_cast<size_t>(B) * N * N;
  float* zn = static_cast<float*>(workspace);
  float* hbuf = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + a256(P * c_p * 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int h = c_p * n;
  if (int e = launch_ln(z, pk + L.lw, pk + L.lb, zn, static_cast<int64_t>(P), c_p, N, 0, st)) return e;
  if (int e = launch_gemm(zn, static_cast<int64_t>(P), c_p, c_p, pk + L.w1, h, c_p, epi(kRelu, pk + L.b1, hbuf, h), st))
    return e;
  Epi e = epi(kResMask, pk + L.b2, out, c_p);
  e.z = add_residual ? z : nullptr;
  e.mask = mask;
  e.N = N;
  return launch_gemm(hbuf, static_cast<int64_t>(P), h, h, pk + L.w2, c_p, h, e, st);
}

}  // namespace gen
}  // namespace gtk

// ---------------------------------------------------------------------------------------
// Linear layers of the reference's modules outside the triangle blocks: the fused
// LayerNorm + linear of its `_C` module and the (gated) projections of `Attention`.
// ---------------------------------------------------------------------------------------
namespace {

int linear_args(const float* x, const float* weight, const float* bias, const float* out, int64_t rows, int64_t D_in,
                int64_t D_out) {
  using namespace gtk;
  if (rows < 1 || !dims_ok(rows, int64_t(1) << 40) || D_in < 1 || D_out < 1 || D_in > (1 << 24) ||
      D_out > (1 << 24) || (D_out + gen::kBN - 1) / gen::kBN > 65535)
    return fail(GTK_ERR_INVALID_ARG, "linear: bad rows / D_in / D_out");
  if (int e = check_ptr(x, "x", 4)) return e;
  if (int e = check_ptr(weight, "weight", 4)) return e;
  if (int e = check_ptr(out, "out", 4)) return e;
  if (bias && (reinterpret_cast<uintptr_t>(bias) & 3)) return fail(GTK_ERR_ALIGNMENT, "bias is misaligned");
  return GTK_OK;
}

int launch_linear(int pro_mode, const float* x, const float* weight, const float* bias, float* out, int64_t rows,
                  int64_t D_in, int64_t D_out, const gtk::gen::Pro& pro, void* stream) {
  using namespace gtk;
  using namespace gtk::gen;
  const Epi e = epi(kStore, bias, out, D_out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int K = static_cast<int>(D_in), n_out = static_cast<int>(D_out);
  // 3xTF32: these entry points promise fp32 results
  if (pro_mode == kProLn)
    return launch_gemm_t<kProLn, 3>(x, rows, K, D_in, weight, n_out, D_in, e, pro, st, "linear gemm_kernel");
  if (pro_mode == kProGate)
    return launch_gemm_t<kProGate, 3>(x, rows, K, D_in, weight, n_out, D_in, e, pro, st, "linear gemm_kernel");
  return launch_gemm_t<kProNone, 3>(x, rows, K, D_in, weight, n_out, D_in, e, pro, st, "linear gemm_kernel");
}

}  // namespace

extern "C" {

int gtk_layernorm_linear(const float* x, const float* gamma, const float* beta, const float* weight,
                         const float* bias, float* out, int64_t rows, int64_t D_in, int64_t D_out, float eps,
                         void* stream) {
  using namespace gtk;
  if (int e = linear_args(x, weight, bias, out, rows, D_in, D_out)) return e;
  if (!(eps >= 0.f) || !std::isfinite(eps)) return fail(GTK_ERR_INVALID_ARG, "layernorm_linear: eps must be >= 0");
  if (int e = check_ptr(gamma, "gamma", 4)) return e;
  if (int e = check_ptr(beta, "beta", 4)) return e;
  if (x == out) return fail(GTK_ERR_INVALID_ARG, "layernorm_linear: out must not alias x");
  if (int e = check_device()) return e;
  gen::Pro pro{};
  pro.gamma = gamma;
  pro.beta = beta;
  pro.eps = eps;
  return launch_linear(gen::kProLn, x, weight, bias, out, rows, D_in, D_out, pro, stream);
}

int gtk_linear(const float* x, const float* gate, const float* weight, const float* bias, float* out, int64_t rows,
               int64_t D_in, int64_t D_out, void* stream) {
  using namespace gtk;
  if (int e = linear_args(x, weight, bias, out, rows, D_in, D_out)) return e;
  if (gate && (reinterpret_cast<uintptr_t>(gate) & 3)) return fail(GTK_ERR_ALIGNMENT, "gate is misaligned");
  if (x == out || (gate && gate == out)) return fail(GTK_ERR_INVALID_ARG, "linear: out must not alias x or gate");
  if (int e = check_device()) return e;
  gen::Pro pro{};
  pro.gate = gate;
  pro.ldg = D_in;
  return launch_linear(gate ? gen::kProGate : gen::kProNone, x, weight, bias, out, rows, D_in, D_out, pro, stream);
}

}  // extern "C"
