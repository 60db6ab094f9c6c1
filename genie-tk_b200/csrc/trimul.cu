// Triangle multiplicative update (AlphaFold2 Algorithms 11/12) on sm_100a.
//
// Reference math: src/genie_tk/triangle_mul.py:103-132 (the PyTorch path, the only
// working implementation of northws/Genie-TK). Three kernels per call:
//
//  K1 trimul_project_kernel  LN_in + the four gated projections (one 128x512x128
//                            tcgen05 GEMM per 128-pair tile) + sigmoid gates + mask;
//                            writes a and b as fp16 channel planes [B, R, C, ld].
//  K2 trimul_contract_kernel the per-channel N x N x N contraction (triangle_mul.py:77-101)
//                            as tcgen05 GEMMs, 128x256 tiles, 4-stage TMA/mbarrier ring;
//                            outgoing uses K-major operands, incoming the MN-major form of
//                            the same planes (no transpose pass). The fp32 accumulator is
//                            stored as fp16 after scaling by `out_scale` (1/K on the forward
//                            path, which keeps |x| far inside the fp16 range).
//  K2e trimul_finish_kernel  LN_out (folded into the GEMM epilogue), linear_z, the output
//                            gate sigmoid(linear_g(LN_in(z))) recomputed from z, and the
//                            optional residual add, written with TMA.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {

// ----------------------------------------------------------------------------------
// Packed weights (built by trimul_pack_kernel from the fp32 module parameters).
// All 16-bit operands are fp16 (tcgen05 kind::f16, fp32 accumulate): each is bounded --
// LayerNorm outputs, fan-in-scaled weights, gated projections, the 1/K-scaled contraction --
// and fp16 keeps 3 more mantissa bits than bf16 at the same tensor-core rate. Conversions
// saturate to the finite fp16 range.
//   W1  fp16 [512][128]: rows 0-127 linear_a_p, 128-255 linear_a_g, 256-383 linear_b_p,
//                        384-511 linear_b_g  (nn.Linear [out, in] = K-major B operand)
//   W2  fp16 [256][128]: rows 0-127 linear_g, 128-255 linear_z * gamma_out (LN_out scale folded)
//   vec fp32: b1[512] (the four projection biases), ln_in_w[128], ln_in_b[128], b_g[128],
//             u[128] = sum_c W2[128+n][c] (fp16-rounded), v[128] = linear_z(beta_out) + b_z.
// LN_out(x) W_z^T + b_z = rstd * (x (W_z*gamma)^T - mu * u) + v for per-pair mean mu, rstd.
// ----------------------------------------------------------------------------------
namespace tmpack {
constexpr size_t kW1 = 0;
constexpr size_t kW2 = 512 * 128 * 2;
constexpr size_t kVec = kW2 + 256 * 128 * 2;
constexpr int kVB1 = 0, kVLnW = 512, kVLnB = 640, kVBg = 768, kVU = 896, kVV = 1024, kVecFloats = 1152;
constexpr size_t kBytes = kVec + kVecFloats * 4;
}  // namespace tmpack

__global__ void trimul_pack_kernel(gtk_trimul_params p, uint8_t* packed) {
  __half* w1 = reinterpret_cast<__half*>(packed + tmpack::kW1);
  __half* w2 = reinterpret_cast<__half*>(packed + tmpack::kW2);
  float* vec = reinterpret_cast<float*>(packed + tmpack::kVec);
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nthreads = gridDim.x * blockDim.x;
  for (int e = tid; e < 512 * 128; e += nthreads) {
    const int r = e >> 7, c = e & 127;
    const float* src = r < 128 ? p.a_p_w : r < 256 ? p.a_g_w : r < 384 ? p.b_p_w : p.b_g_w;
    w1[e] = f16_sat(src[(r & 127) * 128 + c]);
  }
  for (int e = tid; e < 256 * 128; e += nthreads) {
    const int r = e >> 7, c = e & 127;
    const float val = r < 128 ? p.g_w[r * 128 + c] : p.z_w[(r - 128) * 128 + c] * p.ln_out_w[c];
    w2[e] = f16_sat(val);
  }
  for (int e = tid; e < 128; e += nthreads) {
    vec[tmpack::kVB1 + e] = p.a_p_b[e];
    vec[tmpack::kVB1 + 128 + e] = p.a_g_b[e];
    vec[tmpack::kVB1 + 256 + e] = p.b_p_b[e];
    vec[tmpack::kVB1 + 384 + e] = p.b_g_b[e];
    vec[tmpack::kVLnW + e] = p.ln_in_w[e];
    vec[tmpack::kVLnB + e] = p.ln_in_b[e];
    vec[tmpack::kVBg + e] = p.g_b[e];
    float u = 0.f, v = p.z_b[e];
    for (int c = 0; c < 128; ++c) {
      u += __half2float(f16_sat(p.z_w[e * 128 + c] * p.ln_out_w[c]));
      v += p.z_w[e * 128 + c] * p.ln_out_b[c];
    }
    vec[tmpack::kVU + e] = u;
    vec[tmpack::kVV + e] = v;
  }
}

// ----------------------------------------------------------------------------------
// K1: LN_in + gated projections + mask -> a, b planes.
// One CTA per 128-pair tile (pair row r, columns j0..j0+127). 128 threads; thread p owns
// pair j0+p (TMEM lane p). Shared memory: W1 128 KB | A 32 KB | z 64 KB | vec | barriers.
// ----------------------------------------------------------------------------------
namespace k1 {
constexpr uint32_t kW = 0, kA = 131072, kZ = 163840, kBar = 229376;
constexpr uint32_t kSmem = kBar + 64 + 1024;
}  // namespace k1

__global__ void __launch_bounds__(128, 1)
    trimul_project_kernel(const __grid_constant__ CUtensorMap z_map, const __grid_constant__ CUtensorMap w_map,
                          const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                          const float* __restrict__ mask, const float* __restrict__ vec, int N, int rows,
                          uint32_t* status) {
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  uint64_t* zbar = reinterpret_cast<uint64_t*>(smem + k1::kBar);
  uint64_t* wbar = zbar + 1;
  uint64_t* mbar = zbar + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(zbar + 3);
  CtaGuard* guard = reinterpret_cast<CtaGuard*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int j0 = blockIdx.x * 128, r = blockIdx.y, b = blockIdx.z;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(zbar, 1);
    mbar_init(wbar, 1);
    mbar_init(mbar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    mbar_arrive_expect_tx(zbar, 65536);
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_4d(smem + k1::kZ + q * 16384, &z_map, zbar, q * 32, j0, r, b);
    mbar_arrive_expect_tx(wbar, 131072);
#pragma unroll
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll
      for (int rb = 0; rb < 4; ++rb)
        tma_load_2d(smem + k1::kW + kh * 65536 + rb * 16384, &w_map, wbar, kh * 64, rb * 128);
  }

  const int p = tid;
  const int j = j0 + p;
  float mval = 0.f;
  if (j < N) mval = mask ? mask[(static_cast<size_t>(b) * rows + r) * N + j] : 1.f;

  if (mbar_wait(zbar, 0, guard, status, kStatusTimeoutConsumer)) {
    ln_row_to_operand(smem + k1::kZ, smem + k1::kA, p, vec + tmpack::kVLnW, vec + tmpack::kVLnB);
  }
  fence_proxy_async_smem();
  __syncthreads();
  // The z tile is dead now: keep the projection biases there for the epilogue.
  float* sb1 = reinterpret_cast<float*>(smem + k1::kZ);
  reinterpret_cast<float4*>(sb1)[tid] = reinterpret_cast<const float4*>(vec + tmpack::kVB1)[tid];

  if (tid == 0 && !guard->abort) {
    if (mbar_wait(wbar, 0, guard, status, kStatusTimeoutMma)) {
      tc_fence_after();
      const uint32_t idesc = make_idesc_f16(128, 256, 0, 0);
      const uint32_t a0 = smem_u32(smem + k1::kA), w0 = smem_u32(smem + k1::kW);
#pragma unroll
      for (int nh = 0; nh < 2; ++nh)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int kh = ks >> 2, kin = ks & 3;
          const uint64_t ad = make_sdesc(a0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128);
          const uint64_t bd = make_sdesc(w0 + kh * 65536 + nh * 32768 + kin * 32, 16, 1024, Swz::k128);
          umma_ss(tmem + nh * 256, ad, bd, idesc, ks > 0 ? 1u : 0u);
        }
      umma_commit(mbar);
    }
  }
  __syncthreads();
  const bool ok = __all_sync(0xffffffffu, mbar_wait(mbar, 0, guard, status, kStatusTimeoutConsumer));
  tc_fence_after();
  if (ok) {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      __half* stage = reinterpret_cast<__half*>(smem + k1::kW + which * 32768);
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t pr[32], gr[32];
        tmem_ld32(tmem + lane_base + which * 256 + cc * 32, pr);
        tmem_ld32(tmem + lane_base + which * 256 + 128 + cc * 32, gr);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int c = cc * 32 + t;
          const float pv = __uint_as_float(pr[t]) + sb1[which * 256 + c];
          const float gv = __uint_as_float(gr[t]) + sb1[which * 256 + 128 + c];
          stage[c * 128 + p] = f16_sat(pv * sigmoidf_fast(gv) * mval);
        }
      }
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    if (!guard->abort) {
      tma_store_4d(&a_map, smem + k1::kW, j0, 0, r, b);
      tma_store_4d(&b_map, smem + k1::kW + 32768, j0, 0, r, b);
      tma_store_commit();
      tma_store_wait_read();
    } else {
      // drain loads that may still be landing before shared memory is released
      mbar_wait_drain(zbar, 0);
      mbar_wait_drain(wbar, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------------
// K2: per-channel contraction. CTA tile: 128 rows (i) x 256 columns (j) of one (b, c)
// plane; K loop in blocks of 64 through a 4-stage TMA ring. Warp 0 lane 0 = TMA producer,
// warp 1 lane 0 = MMA issuer (TMEM accumulator, 256 columns), all 4 warps = epilogue.
// ----------------------------------------------------------------------------------
namespace k2 {
constexpr int kStages = 4;
constexpr uint32_t kStageBytes = 49152;  // A 128x64 (16 KB) + B 256x64 (32 KB)
constexpr uint32_t kBar = kStages * kStageBytes;
constexpr uint32_t kSmem = kBar + 128 + 1024;
}  // namespace k2

template <bool kOutgoing>
__global__ void __launch_bounds__(128, 1)
    trimul_contract_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                           const __grid_constant__ CUtensorMap x_map, int C, int K, float out_scale,
                           uint32_t* status) {
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + k2::kBar);
  uint64_t* empty = full + k2::kStages;
  uint64_t* done = empty + k2::kStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);
  CtaGuard* guard = reinterpret_cast<CtaGuard*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int jt = blockIdx.x, it = blockIdx.y;
  const int c = blockIdx.z % C, b = blockIdx.z / C;
  const int KB = (K + 63) / 64;

  if (tid == 0) {
    guard->abort = 0;
    for (int s = 0; s < k2::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0 && lane == 0) {
    int issued = 0;
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % k2::kStages;
      if (kb >= k2::kStages && !mbar_wait(&empty[s], ((kb / k2::kStages) - 1) & 1, guard, status,
                                          kStatusTimeoutProducer))
        break;
      mbar_arrive_expect_tx(&full[s], k2::kStageBytes);
      uint8_t* sa = smem + s * k2::kStageBytes;
      uint8_t* sb = sa + 16384;
      if (kOutgoing) {
        tma_load_4d(sa, &a_map, &full[s], kb * 64, c, it * 128, b);
        tma_load_4d(sb, &b_map, &full[s], kb * 64, c, jt * 256, b);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) tma_load_4d(sa + h * 8192, &a_map, &full[s], it * 128 + h * 64, c, kb * 64, b);
#pragma unroll
        for (int q = 0; q < 4; ++q) tma_load_4d(sb + q * 8192, &b_map, &full[s], jt * 256 + q * 64, c, kb * 64, b);
      }
      ++issued;
    }
    if (guard->abort) {
      // drain: wait for every load this thread issued that may still be in flight
      for (int kb = (issued > k2::kStages ? issued - k2::kStages : 0); kb < issued; ++kb)
        mbar_wait_drain(&full[kb % k2::kStages], (kb / k2::kStages) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = make_idesc_f16(128, 256, kOutgoing ? 0u : 1u, kOutgoing ? 0u : 1u);
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % k2::kStages;
      if (!mbar_wait(&full[s], (kb / k2::kStages) & 1, guard, status, kStatusTimeoutMma)) break;
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * k2::kStageBytes);
      const uint32_t sb = sa + 16384;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint64_t ad, bd;
        if (kOutgoing) {
          ad = make_sdesc(sa + ks * 32, 16, 1024, Swz::k128);
          bd = make_sdesc(sb + ks * 32, 16, 1024, Swz::k128);
        } else {
          ad = make_sdesc(sa + ks * 2048, 8192, 1024, Swz::k128);
          bd = make_sdesc(sb + ks * 2048, 8192, 1024, Swz::k128);
        }
        umma_ss(tmem, ad, bd, idesc, (kb | ks) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  }

  const bool waited = mbar_wait(done, 0, guard, status, kStatusTimeoutConsumer);
  const bool ok = __all_sync(0xffffffffu, waited && !guard->abort);
  tc_fence_after();
  if (ok) {
    const int p = tid;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll 1
    for (int cc = 0; cc < 8; ++cc) {
      uint32_t v[32];
      tmem_ld32(tmem + lane_base + cc * 32, v);
      tmem_wait_ld();
      uint8_t* box = smem + (cc >> 1) * 16384;
      const int chb = (cc & 1) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 o;
        o.x = pack_f16x2(__uint_as_float(v[u * 8 + 0]) * out_scale, __uint_as_float(v[u * 8 + 1]) * out_scale);
        o.y = pack_f16x2(__uint_as_float(v[u * 8 + 2]) * out_scale, __uint_as_float(v[u * 8 + 3]) * out_scale);
        o.z = pack_f16x2(__uint_as_float(v[u * 8 + 4]) * out_scale, __uint_as_float(v[u * 8 + 5]) * out_scale);
        o.w = pack_f16x2(__uint_as_float(v[u * 8 + 6]) * out_scale, __uint_as_float(v[u * 8 + 7]) * out_scale);
        sts_u4(box + swz128(p, chb + u), o);
      }
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0 && ok && !guard->abort) {
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_store_4d(&x_map, smem + q * 16384, jt * 256 + q * 64, c, it * 128, b);
    tma_store_commit();
    tma_store_wait_read();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ----------------------------------------------------------------------------------
// K2e: LN_out + linear_z + output gate (+ residual). One CTA per 128-pair tile.
// Shared memory: W2 64 KB | z 64 KB | x 32 KB | LN_in(z) 32 KB | vec 2.5 KB | barriers.
// TMEM: cols 0-127 gate pre-activation G, cols 128-255 U = x (W_z*gamma)^T.
// ----------------------------------------------------------------------------------
namespace k2e {
constexpr uint32_t kW = 0, kZ = 65536, kX = 131072, kA = 163840, kVec = 196608, kBar = 196608 + 2560;
constexpr uint32_t kSmem = kBar + 64 + 1024;
}  // namespace k2e

__global__ void __launch_bounds__(128, 1)
    trimul_finish_kernel(const __grid_constant__ CUtensorMap z_map, const __grid_constant__ CUtensorMap w_map,
                         const __grid_constant__ CUtensorMap x_map, const __grid_constant__ CUtensorMap out_map,
                         const float* __restrict__ vec, int add_residual, float x_scale, uint32_t* status) {
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  uint64_t* lbar = reinterpret_cast<uint64_t*>(smem + k2e::kBar);
  uint64_t* mbar = lbar + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(lbar + 2);
  CtaGuard* guard = reinterpret_cast<CtaGuard*>(tslot + 1);
  float* svec = reinterpret_cast<float*>(smem + k2e::kVec);  // b_g | u | v | ln_w | ln_b
  const int tid = threadIdx.x, warp = tid >> 5;
  const int j0 = blockIdx.x * 128, r = blockIdx.y, b = blockIdx.z;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(lbar, 1);
    mbar_init(mbar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  svec[tid] = vec[tmpack::kVBg + tid];
  svec[128 + tid] = vec[tmpack::kVU + tid];
  svec[256 + tid] = vec[tmpack::kVV + tid];
  svec[384 + tid] = vec[tmpack::kVLnW + tid];
  svec[512 + tid] = vec[tmpack::kVLnB + tid];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    mbar_arrive_expect_tx(lbar, 65536 + 65536 + 32768);
#pragma unroll
    for (int kh = 0; kh < 2; ++kh) tma_load_2d(smem + k2e::kW + kh * 32768, &w_map, lbar, kh * 64, 0);
#pragma unroll
    for (int q = 0; q < 4; ++q) tma_load_4d(smem + k2e::kZ + q * 16384, &z_map, lbar, q * 32, j0, r, b);
#pragma unroll
    for (int h = 0; h < 2; ++h) tma_load_4d(smem + k2e::kX + h * 16384, &x_map, lbar, j0 + h * 64, 0, r, b);
  }
  const int p = tid;
  float mu_x = 0.f, rstd_x = 0.f;
  if (mbar_wait(lbar, 0, guard, status, kStatusTimeoutConsumer)) {
    ln_row_to_operand(smem + k2e::kZ, smem + k2e::kA, p, svec + 384, svec + 512);
    // LN_out statistics over the 128 channels of pair p, read from the [c][j] x tile.
    const uint8_t* xb = smem + k2e::kX + (p >> 6) * 16384;
    const int pj = p & 63;
    float s = 0.f;
#pragma unroll 8
    for (int c = 0; c < 128; ++c) {
      const uint16_t bits = *reinterpret_cast<const uint16_t*>(xb + swz128(c, pj >> 3) + (pj & 7) * 2);
      s += __half2float(__ushort_as_half(bits));
    }
    mu_x = s * (1.f / 128.f);
    float ss = 0.f;
#pragma unroll 8
    for (int c = 0; c < 128; ++c) {
      const uint16_t bits = *reinterpret_cast<const uint16_t*>(xb + swz128(c, pj >> 3) + (pj & 7) * 2);
      const float d = __half2float(__ushort_as_half(bits)) - mu_x;
      ss += d * d;
    }
    // x is stored scaled by x_scale; LN(x) = LN_eps*s^2(x * s), so the eps scales with it.
    rstd_x = rsqrtf(ss * (1.f / 128.f) + 1e-5f * x_scale * x_scale);
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0 && !guard->abort) {
    tc_fence_after();
    const uint32_t a0 = smem_u32(smem + k2e::kA), w0 = smem_u32(smem + k2e::kW), x0 = smem_u32(smem + k2e::kX);
    const uint32_t id_g = make_idesc_f16(128, 128, 0, 0);
    const uint32_t id_u = make_idesc_f16(128, 128, 1, 0);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int kh = ks >> 2, kin = ks & 3;
      umma_ss(tmem, make_sdesc(a0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128),
              make_sdesc(w0 + kh * 32768 + kin * 32, 16, 1024, Swz::k128), id_g, ks > 0 ? 1u : 0u);
    }
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int kh = ks >> 2, kin = ks & 3;
      umma_ss(tmem + 128, make_sdesc(x0 + ks * 2048, 16384, 1024, Swz::k128),
              make_sdesc(w0 + kh * 32768 + 16384 + kin * 32, 16, 1024, Swz::k128), id_u, ks > 0 ? 1u : 0u);
    }
    umma_commit(mbar);
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(mbar, 0, guard, status, kStatusTimeoutConsumer));
  tc_fence_after();
  if (ok) {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t g[32], u[32];
      tmem_ld32(tmem + lane_base + cc * 32, g);
      tmem_ld32(tmem + lane_base + 128 + cc * 32, u);
      tmem_wait_ld();
      uint8_t* zq = smem + k2e::kZ + cc * 16384;  // channels cc*32 .. cc*32+31
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        float4 zv = lds_f4(zq + swz128(p, ch));
        float res[4] = {zv.x, zv.y, zv.z, zv.w};
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = ch * 4 + e, n = cc * 32 + t;
          const float gate = sigmoidf_fast(__uint_as_float(g[t]) + svec[n]);
          const float y = (rstd_x * (__uint_as_float(u[t]) - mu_x * svec[128 + n]) + svec[256 + n]) * gate;
          o[e] = add_residual ? y + res[e] : y;
        }
        *reinterpret_cast<float4*>(zq + swz128(p, ch)) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    if (ok && !guard->abort) {
#pragma unroll
      for (int q = 0; q < 4; ++q) tma_store_4d(&out_map, smem + k2e::kZ + q * 16384, q * 32, j0, r, b);
      tma_store_commit();
      tma_store_wait_read();
    } else {
      mbar_wait_drain(lbar, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ----------------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------------

}  // namespace gtk

using namespace gtk;

extern "C" {

size_t gtk_trimul_packed_bytes(int c_z, int c_hidden) {
  if (c_z != 128 || c_hidden != 128) return 0;
  return tmpack::kBytes;
}

int gtk_trimul_pack(const gtk_trimul_params* params, int c_z, int c_hidden, void* packed, size_t packed_bytes,
                    void* stream) {
  if (c_z != 128 || c_hidden != 128)
    return fail(GTK_ERR_UNSUPPORTED, "trimul: only c_z = c_hidden = 128 is implemented");
  if (!params) return fail(GTK_ERR_INVALID_ARG, "params is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < tmpack::kBytes) return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  const float* const* pp = reinterpret_cast<const float* const*>(params);
  for (int i = 0; i < 16; ++i)
    if (!pp[i]) return fail(GTK_ERR_INVALID_ARG, "a trimul parameter pointer is NULL");
  if (int e = check_device()) return e;
  trimul_pack_kernel<<<64, 256, 0, static_cast<cudaStream_t>(stream)>>>(*params, static_cast<uint8_t*>(packed));
  return check_launch("trimul_pack_kernel");
}

int64_t gtk_plane_pitch(int64_t N) { return static_cast<int64_t>(round_up(static_cast<uint64_t>(N), 8)); }

size_t gtk_trimul_workspace_bytes(int64_t B, int64_t N, int c_z, int c_hidden) {
  if (c_z != 128 || c_hidden != 128 || B < 1 || N < 1) return 0;
  const size_t plane = round_up(static_cast<size_t>(B) * N * 128 * gtk_plane_pitch(N) * 2, 256);
  return 3 * plane;
}

int gtk_trimul_project(const float* z, const float* mask, const void* packed, void* a_planes, void* b_planes,
                       int64_t ld, int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream) {
  if (!dims_ok(B, 65535) || !dims_ok(rows, 65535) || !dims_ok(N, 1 << 20))
    return fail(GTK_ERR_INVALID_ARG, "trimul_project: bad B/rows/N");
  if (ld < N || ld % 8) return fail(GTK_ERR_INVALID_ARG, "trimul_project: plane pitch must be >= N and a multiple of 8");
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_ptr(a_planes, "a_planes")) return e;
  if (int e = check_ptr(b_planes, "b_planes")) return e;
  if (int e = check_device()) return e;
  CUtensorMap zm, wm, am, bm;
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  if (int e = make_pair_map(&zm, z, B, rows, N, false)) return e;
  if (int e = make_weight_map(&wm, pk + tmpack::kW1, 512, 128)) return e;
  if (int e = make_plane_map(&am, a_planes, B, rows, 128, N, ld, 128, 128, 1, 0)) return e;
  if (int e = make_plane_map(&bm, b_planes, B, rows, 128, N, ld, 128, 128, 1, 0)) return e;
  if (int e = ensure_smem(reinterpret_cast<const void*>(trimul_project_kernel), k1::kSmem)) return e;
  dim3 grid(static_cast<unsigned>((N + 127) / 128), static_cast<unsigned>(rows), static_cast<unsigned>(B));
  trimul_project_kernel<<<grid, 128, k1::kSmem, static_cast<cudaStream_t>(stream)>>>(
      zm, wm, am, bm, mask, reinterpret_cast<const float*>(pk + tmpack::kVec), static_cast<int>(N),
      static_cast<int>(rows), status);
  return check_launch("trimul_project_kernel");
}

int gtk_trimul_contract(int outgoing, const void* a_planes, const void* b_planes, void* x_planes, int64_t B,
                        int64_t C, int64_t M, int64_t Nj, int64_t K, int64_t lda, int64_t ldb, int64_t ldx,
                        float out_scale, uint32_t* status, void* stream) {
  if (!dims_ok(B) || !dims_ok(C) || !dims_ok(M) || !dims_ok(Nj) || !dims_ok(K) || B * C > 65535 * 1024)
    return fail(GTK_ERR_INVALID_ARG, "trimul_contract: bad sizes");
  if (lda % 8 || ldb % 8 || ldx % 8) return fail(GTK_ERR_ALIGNMENT, "trimul_contract: pitches must be multiples of 8");
  if (outgoing ? (lda < K || ldb < K) : (lda < M || ldb < Nj)) return fail(GTK_ERR_INVALID_ARG, "pitch too small");
  if (ldx < Nj) return fail(GTK_ERR_INVALID_ARG, "trimul_contract: ldx < Nj");
  if (int e = check_ptr(a_planes, "a_planes")) return e;
  if (int e = check_ptr(b_planes, "b_planes")) return e;
  if (int e = check_ptr(x_planes, "x_planes")) return e;
  if (int e = check_device()) return e;
  CUtensorMap am, bm, xm;
  if (outgoing) {
    if (int e = make_plane_map(&am, a_planes, B, M, C, K, lda, 64, 1, 128, 128)) return e;
    if (int e = make_plane_map(&bm, b_planes, B, Nj, C, K, ldb, 64, 1, 256, 128)) return e;
  } else {
    if (int e = make_plane_map(&am, a_planes, B, K, C, M, lda, 64, 1, 64, 128)) return e;
    if (int e = make_plane_map(&bm, b_planes, B, K, C, Nj, ldb, 64, 1, 64, 128)) return e;
  }
  if (int e = make_plane_map(&xm, x_planes, B, M, C, Nj, ldx, 64, 1, 128, 128)) return e;
  const void* kern = outgoing ? reinterpret_cast<const void*>(trimul_contract_kernel<true>)
                              : reinterpret_cast<const void*>(trimul_contract_kernel<false>);
  if (int e = ensure_smem(kern, k2::kSmem)) return e;
  dim3 grid(static_cast<unsigned>((Nj + 255) / 256), static_cast<unsigned>((M + 127) / 128),
            static_cast<unsigned>(B * C));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (outgoing)
    trimul_contract_kernel<true><<<grid, 128, k2::kSmem, st>>>(am, bm, xm, static_cast<int>(C), static_cast<int>(K),
                                                                out_scale, status);
  else
    trimul_contract_kernel<false><<<grid, 128, k2::kSmem, st>>>(am, bm, xm, static_cast<int>(C),
                                                                 static_cast<int>(K), out_scale, status);
  return check_launch("trimul_contract_kernel");
}

int gtk_trimul_finish(const float* z, const void* x_planes, int64_t ldx, float x_scale, const void* packed,
                      float* out, int add_residual, int64_t B, int64_t rows, int64_t N, uint32_t* status,
                      void* stream) {
  if (!dims_ok(B, 65535) || !dims_ok(rows, 65535) || !dims_ok(N, 1 << 20))
    return fail(GTK_ERR_INVALID_ARG, "trimul_finish: bad B/rows/N");
  if (ldx < N || ldx % 8) return fail(GTK_ERR_INVALID_ARG, "trimul_finish: bad plane pitch");
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(out, "out")) return e;
  if (int e = check_ptr(x_planes, "x_planes")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_device()) return e;
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  CUtensorMap zm, wm, xm, om;
  if (int e = make_pair_map(&zm, z, B, rows, N, false)) return e;
  if (int e = make_weight_map(&wm, pk + tmpack::kW2, 256, 256)) return e;
  if (int e = make_plane_map(&xm, x_planes, B, rows, 128, N, ldx, 64, 128, 1, 128)) return e;
  if (int e = make_pair_map(&om, out, B, rows, N, false)) return e;
  if (int e = ensure_smem(reinterpret_cast<const void*>(trimul_finish_kernel), k2e::kSmem)) return e;
  dim3 grid(static_cast<unsigned>((N + 127) / 128), static_cast<unsigned>(rows), static_cast<unsigned>(B));
  trimul_finish_kernel<<<grid, 128, k2e::kSmem, static_cast<cudaStream_t>(stream)>>>(
      zm, wm, xm, om, reinterpret_cast<const float*>(pk + tmpack::kVec), add_residual, x_scale, status);
  return check_launch("trimul_finish_kernel");
}

int gtk_trimul_forward(int outgoing, const float* z, const float* mask, const void* packed, float* out,
                       int add_residual, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_z,
                       int c_hidden, uint32_t* status, void* stream) {
  if (c_z != 128 || c_hidden != 128)
    return fail(GTK_ERR_UNSUPPORTED, "trimul: only c_z = c_hidden = 128 is implemented");
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535)) return fail(GTK_ERR_INVALID_ARG, "trimul: bad B/N");
  const size_t need = gtk_trimul_workspace_bytes(B, N, c_z, c_hidden);
  if (workspace_bytes < need) return fail(GTK_ERR_WORKSPACE, "trimul: workspace too small");
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  const int64_t ld = gtk_plane_pitch(N);
  const size_t plane = need / 3;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* ap = ws;
  void* bp = ws + plane;
  void* xp = ws + 2 * plane;
  if (int e = gtk_trimul_project(z, mask, packed, ap, bp, ld, B, N, N, status, stream)) return e;
  const float xs = 1.0f / static_cast<float>(N);
  if (int e = gtk_trimul_contract(outgoing, ap, bp, xp, B, 128, N, N, N, ld, ld, ld, xs, status, stream)) return e;
  return gtk_trimul_finish(z, xp, ld, xs, packed, out, add_residual, B, N, N, status, stream);
}

}  // extern "C"
