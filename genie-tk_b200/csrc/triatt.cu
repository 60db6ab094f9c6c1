// Triangle attention around the starting / ending node (AlphaFold2 Algorithms 13/14)
// on sm_100a.
//
// Reference math: src/genie_tk/triangle_attention.py:100-143 and the gated attention of
// src/genie_tk/primitives.py:114-178. For every row i of the (possibly transposed) pair
// tensor, H independent attentions over the N positions of that row:
//   s[j,k] = q_ij.k_ik / sqrt(d) + inf*(mask[i,k]-1) + bias[h,j,k],  bias = LN(z)[j,k].w_h
//   o[i,j] = softmax_k(s) v_i,  update = linear_o(o * sigmoid(linear_g(LN(z))))
// Three kernels per call:
//  K3 triatt_project_kernel LN + one 128x512x128 tcgen05 GEMM per 128-pair tile for q
//                           (pre-scaled by log2(e)/sqrt(d)), k, v and the gate, plus the
//                           4-head triangle bias on CUDA cores from the fp32 LN output.
//  K4 triatt_core_kernel    flash-style attention: S = Q K^T and O += P V on tcgen05 with
//                           S, P and O in TMEM, online softmax in base 2 with the bias
//                           and mask bias folded into the logits; the N^3 score tensor is
//                           never formed. A CTA owns one 128-query tile of one head for 4
//                           rows i, so each bias tile loaded to shared memory serves 4 rows.
//                           The epilogue normalises O and applies the gate.
//  K4e triatt_finish_kernel linear_o (tcgen05) + bias + optional residual add.
// The ending node is the starting node on z^T: K3 reads and K4e writes the pair tensor
// through transposed TMA descriptors, and K4 reads the mask with swapped strides.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"
#include "general.h"

namespace gtk {

constexpr int kHeads = 4;
constexpr int kHeadDim = 32;
constexpr float kLog2e = 1.4426950408889634f;

// ----------------------------------------------------------------------------------
// Packed weights (fp16 operands, fp32 vectors):
//   W3 fp16 [512][128]: rows 0-127 linear_q * log2(e)/sqrt(d), 128-255 linear_k,
//                       256-383 linear_v, 384-511 linear_g / 2
//   W4 fp16 [128][128]: linear_o
//   vec fp32: ln_w[128], ln_b[128], w_bias[4][128] * log2(e), b_g[128] / 2, b_o[128]
// ----------------------------------------------------------------------------------
namespace tapack {
constexpr size_t kW3 = 0;
constexpr size_t kW4 = 512 * 128 * 2;
constexpr size_t kVec = kW4 + 128 * 128 * 2;
constexpr int kVLnW = 0, kVLnB = 128, kVWb = 256, kVBg = 768, kVBo = 896, kVecFloats = 1024;
constexpr size_t kBytes = kVec + kVecFloats * 4;
}  // namespace tapack

// Packs the parameters of 4 heads of head_dim d <= 32 (c_hidden = 4d) into the tuned
// layout of 4 heads of 32: hidden channel h*32 + e is the module's channel h*d + e for e < d
// and zero above (zero rows of W_q / W_k / W_v / W_g and b_g, zero columns of W_o), so the
// padded q, k, v, gated output and their products are exact. q carries log2 e / sqrt(d).
__global__ void triatt_pack_kernel(gtk_triatt_params p, uint8_t* packed, float q_scale, int d) {
  __half* w3 = reinterpret_cast<__half*>(packed + tapack::kW3);
  __half* w4 = reinterpret_cast<__half*>(packed + tapack::kW4);
  float* vec = reinterpret_cast<float*>(packed + tapack::kVec);
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nthreads = gridDim.x * blockDim.x;
  const int hd = 4 * d;
  auto src_row = [d](int r) { return (r & 31) < d ? (r >> 5) * d + (r & 31) : -1; };  // padded -> module channel
  for (int e = tid; e < 512 * 128; e += nthreads) {
    const int r = e >> 7, c = e & 127;
    const int sr = src_row(r & 127);
    float v = 0.f;
    if (sr >= 0) {
      if (r < 128) v = p.q_w[sr * 128 + c] * q_scale;
      else if (r < 256) v = p.k_w[sr * 128 + c];
      else if (r < 384) v = p.v_w[sr * 128 + c];
      else v = 0.5f * p.g_w[sr * 128 + c];  // sigmoid(x) = (1 + tanh(x/2)) / 2
    }
    w3[e] = f16_sat(v);
  }
  for (int e = tid; e < 128 * 128; e += nthreads) {
    const int o = e >> 7, sc = src_row(e & 127);
    w4[e] = f16_sat(sc >= 0 ? p.o_w[o * hd + sc] : 0.f);
  }
  for (int e = tid; e < 128; e += nthreads) {
    const int sr = src_row(e);
    vec[tapack::kVLnW + e] = p.ln_w[e];
    vec[tapack::kVLnB + e] = p.ln_b[e];
    vec[tapack::kVBg + e] = sr >= 0 ? 0.5f * p.g_b[sr] : 0.f;
    vec[tapack::kVBo + e] = p.o_b[e];
    for (int h = 0; h < kHeads; ++h) vec[tapack::kVWb + h * 128 + e] = p.bias_w[h * 128 + e] * kLog2e;
  }
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Sum of four per-lane values over the warp, transposed: afterwards lanes 8h..8h+7 hold
// the warp total of value h (6 shuffles instead of 4 x 5).
__device__ __forceinline__ float warp_sum4_transposed(float v0, float v1, float v2, float v3, int lane) {
  const bool hi16 = lane & 16;
  float a = hi16 ? v2 : v0, b = hi16 ? v3 : v1;          // keep {0,1} or {2,3}
  const float sa = hi16 ? v0 : v2, sb = hi16 ? v1 : v3;  // send the other pair
  a += __shfl_xor_sync(0xffffffffu, sa, 16);
  b += __shfl_xor_sync(0xffffffffu, sb, 16);
  const bool hi8 = lane & 8;
  float c = hi8 ? b : a;
  c += __shfl_xor_sync(0xffffffffu, hi8 ? a : b, 8);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

// ----------------------------------------------------------------------------------
// K3: persistent LN + q/k/v/g projections + triangle bias. Tile = 128 consecutive pairs
// (b, row i of the problem, j0..j0+127); CTAs loop over tiles. 512 threads:
//   warps 0-7  LayerNorm producers, two threads per pair row (64 channels each): one pass
//              reads the staged z tile into registers and releases it, then the fp16
//              operand A and the four triangle-bias dot products of the fp32 LN output
//              (stored bf16, times log2 e) are formed; statistics and dot products combine
//              with one shuffle each (a warp-per-row version spent ~700 cycles per row in
//              dependent shuffle chains; one thread per row with three passes kept the z
//              buffer busy through the whole LayerNorm).
//              Thread 0 is also the TMA producer and MMA issuer: the 128 KB of weights are
//              loaded once; each tile's 128 x 128 fp32 z block (z^T for the ending node,
//              through the transposed descriptor) arrives by TMA, refilled as soon as all
//              producers have read it; after writing its part of A it issues the tile's
//              MMAs. No warp is spent on issuing alone, so sixteen warps keep 128 registers
//              per thread (a seventeen-warp launch is allocated like twenty warps, 96
//              registers, and spills).
//   warps 8-15 epilogue, thread = pair (TMEM lane quarter = warp % 4); warps 8-11 take heads
//              0-1 and warps 12-15 heads 2-3 of TMEM half 0 (q, k), then of half 1 (v and
//              the gate), in 16-column chunks whose TMEM loads run one chunk ahead; each
//              chunk is one 32-byte store per output row (64 B per head row, 256 B gate row).
//              Two warps per scheduler: with one, a K1 epilogue of the same shape was
//              latency-bound (clock64 trace).
// TMEM: half 0 = (q, k) columns 0-255, half 1 = (v, g) columns 256-511; the epilogue of
// half 0 overlaps the MMAs of half 1, and the next tile's LayerNorm and z load overlap both.
// Gate: W3's gate rows and b_g carry a factor 1/2, sigmoid(x) = (1 + tanh(x/2)) / 2.
// Shared memory: W3 128 KB | z 64 KB | A 32 KB | b_g/2 512 B | barriers.
// Rows: the tile grid covers `rows` problem rows i (all N when unsharded; one shard's rows
// under row sharding, which only the starting orientation supports).
// Outputs: q, k, v fp16 [B*rows(i)][H][N(j)][32]; g fp16 [B*rows*N][128]; bias bf16
// [N(row)][B][H][ldn], rows row0.. row0+rows-1 written here (row-major over the problem
// row, so that the shards of a row-sharded run are contiguous and can be all-gathered in
// place; log2 units; bf16 keeps the attention core's shared-memory reads of the
// bias tile at 256 B per query row and step, and widens with one integer op).
// ----------------------------------------------------------------------------------
namespace k3 {
constexpr int kThreads = 512;
// Parameters staged in shared memory: gamma / beta fp32 [8 chunks][2 halves][8] each,
// the bias weights fp16 [8 chunks][4 heads][2 halves][8], b_g / 2 fp32 [128].
constexpr uint32_t kW = 0, kZ = 131072, kA = 196608, kLnW = 229376, kLnB = 229888, kWb = 230400, kBg = 231424,
                   kBar = 231936;
// No alignment slack: the kernel requires a 1024-aligned dynamic shared-memory base (it
// checks, and reports GTK_STATUS bit 4 without touching memory otherwise).
constexpr uint32_t kSmem = kBar + 128;
static_assert(kSmem <= 232448, "K3 shared memory");
}  // namespace k3

struct K3Bars {
  uint64_t wbar;
  uint64_t z_full, z_empty;
  uint64_t a_full, a_empty;
  uint64_t d_full[2], d_empty[2];
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K3Bars) <= 128, "K3 barrier block");

__global__ void __launch_bounds__(k3::kThreads, 1)
    triatt_project_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap z_map,
                          const float* __restrict__ vec, __half* __restrict__ q_out, __half* __restrict__ k_out,
                          __half* __restrict__ v_out, __half* __restrict__ g_out, __nv_bfloat16* __restrict__ bias,
                          int N, int rows, int B, int row0, int ldn, int n_jt, int n_tiles, uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t dsmem[];
  if (smem_u32(dsmem) & 1023u) {  // uniform across the CTA: every thread leaves here
    if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadLaunch);
    return;
  }
  uint8_t* smem = dsmem;
  K3Bars* bars = reinterpret_cast<K3Bars*>(smem + k3::kBar);
  CtaGuard* guard = &bars->guard;
  float* lnw_s = reinterpret_cast<float*>(smem + k3::kLnW);
  float* lnb_s = reinterpret_cast<float*>(smem + k3::kLnB);
  __half* wb_s = reinterpret_cast<__half*>(smem + k3::kWb);
  float* bg_s = reinterpret_cast<float*>(smem + k3::kBg);  // b_g / 2
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
  if (tid < 128) {
    const int c = tid, hf = c >> 6, ch = (c & 63) >> 3, e = c & 7;  // channel c = 64 hf + 8 ch + e
    bg_s[c] = vec[tapack::kVBg + c];
    lnw_s[(ch * 2 + hf) * 8 + e] = vec[tapack::kVLnW + c];
    lnb_s[(ch * 2 + hf) * 8 + e] = vec[tapack::kVLnB + c];
#pragma unroll
    for (int h = 0; h < kHeads; ++h)
      wb_s[((ch * kHeads + h) * 2 + hf) * 8 + e] = __float2half_rn(vec[tapack::kVWb + h * 128 + c]);
  }
  if (warp == 8) {
    tmem_alloc(&bars->tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;

  if (warp < 8) {
    // ---------- LayerNorm + bias producers (two threads per pair row); thread 0 also issues ----------
    // One pass reads the row half from the staged, 128-B-swizzled z tile into registers and
    // releases the tile (the next tile's load overlaps the rest); statistics and the four
    // triangle-bias dot products combine with one shuffle each. gamma, beta and the bias
    // weights are read from shared memory, laid out so that the two row halves of a warp
    // read adjacent 16-byte blocks (one wavefront per load). (As L1-served global loads they
    // missed: the epilogue's 128 KB of stores per tile pass through a small L1, and the
    // LayerNorm's operand phase took ~11,500 cycles per tile, clock64 trace.)
    const int p = warp * 16 + (lane >> 1), half = lane & 1;
    auto load_z = [&](int tile) {
      const int jt = tile % n_jt, bi = tile / n_jt;
      const int i = bi % rows, b = bi / rows;
      mbar_arrive_expect_tx(&bars->z_full, 65536);
#pragma unroll
      for (int q = 0; q < 4; ++q) tma_load_4d(smem + k3::kZ + q * 16384, &z_map, &bars->z_full, q * 32, jt * 128, i, b);
    };
    int loaded = 0;  // z tiles requested (thread 0)
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars->wbar, 131072);
#pragma unroll
      for (int kh = 0; kh < 2; ++kh)
#pragma unroll
        for (int rb = 0; rb < 4; ++rb)
          tma_load_2d(smem + k3::kW + kh * 65536 + rb * 16384, &w_map, &bars->wbar, kh * 64, rb * 128);
      load_z(blockIdx.x);  // the grid never exceeds the tile count
      loaded = 1;
    }
    bool ok = true;
    uint32_t sat = 0;  // a LayerNorm output beyond the fp16 range was clamped
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int jt = tile % n_jt, bi = tile / n_jt;
      const int i = bi % rows, b = bi / rows, j0 = jt * 128;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->z_full, it & 1, guard, status, kStatusTimeoutProducer));
      if (!ok) break;
      const uint8_t* zt = smem + k3::kZ;
      float v[64];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float4 t = lds_f4(zt + (2 * half + q) * 16384 + swz128(p, ch));
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
      float bacc[kHeads] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int c = ch * 8;
        const float* lw = lnw_s + (ch * 2 + half) * 8;
        const float* lb = lnb_s + (ch * 2 + half) * 8;
        const float4 w0 = *reinterpret_cast<const float4*>(lw), w1 = *reinterpret_cast<const float4*>(lw + 4);
        const float4 b0 = *reinterpret_cast<const float4*>(lb), b1 = *reinterpret_cast<const float4*>(lb + 4);
        const float y[8] = {(v[c + 0] - mean) * rstd * w0.x + b0.x, (v[c + 1] - mean) * rstd * w0.y + b0.y,
                            (v[c + 2] - mean) * rstd * w0.z + b0.z, (v[c + 3] - mean) * rstd * w0.w + b0.w,
                            (v[c + 4] - mean) * rstd * w1.x + b1.x, (v[c + 5] - mean) * rstd * w1.y + b1.y,
                            (v[c + 6] - mean) * rstd * w1.z + b1.z, (v[c + 7] - mean) * rstd * w1.w + b1.w};
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          const uint4 u = *reinterpret_cast<const uint4*>(wb_s + ((ch * kHeads + h) * 2 + half) * 8);
          const float2 u0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
          const float2 u1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
          const float2 u2 = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
          const float2 u3 = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
          bacc[h] += y[0] * u0.x + y[1] * u0.y + y[2] * u1.x + y[3] * u1.y + y[4] * u2.x + y[5] * u2.y +
                     y[6] * u3.x + y[7] * u3.y;
        }
        uint4 o;
        o.x = pack_f16x2_chk(y[0], y[1], sat);
        o.y = pack_f16x2_chk(y[2], y[3], sat);
        o.z = pack_f16x2_chk(y[4], y[5], sat);
        o.w = pack_f16x2_chk(y[6], y[7], sat);
        sts_u4(smem + k3::kA + half * 16384 + swz128(p, ch), o);
      }
#pragma unroll
      for (int h = 0; h < kHeads; ++h) bacc[h] += __shfl_xor_sync(0xffffffffu, bacc[h], 1);
      const int j = j0 + p;
      if (half == 0 && j < N) {
#pragma unroll
        for (int h = 0; h < kHeads; ++h)
          bias[((static_cast<size_t>(row0 + i) * B + b) * kHeads + h) * ldn + j] = __float2bfloat16_rn(bacc[h]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->a_full);
      if (warp == 0) {
        // thread 0: the tile's MMAs, half h once the epilogue has drained half h of the
        // previous tile
        bool mw = true;
        if (lane == 0) {
          const uint32_t idesc = make_idesc_f16(128, 256, 0, 0);
          const uint32_t w0 = smem_u32(smem + k3::kW), a0 = smem_u32(smem + k3::kA);
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
    flag_saturation(sat, status);
    if (!ok && tid == 0) {
      // abort: wait (bounded) for this thread's MMAs and TMA loads still in flight
      umma_commit(&bars->drain);
      mbar_wait_drain(&bars->drain, 0);
      if (loaded > 0) mbar_wait_drain(&bars->z_full, (loaded - 1) & 1);
      mbar_wait_drain(&bars->wbar, 0);
    }
  } else {
    // ---------- epilogue: thread = pair; heads 2*hh, 2*hh+1 of TMEM half 0 (q, k), then 1 (v, gate) ----------
    const int q4 = warp & 3, hh = (warp - 8) >> 2;
    const int p = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t sat = 0;  // a q / k / v value beyond the fp16 range was clamped
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int jt = tile % n_jt, bi = tile / n_jt;
      const int j = jt * 128 + p;
      const bool valid = j < N;
      bool ok = true;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[h], it & 1, guard, status, kStatusTimeoutConsumer));
        if (!ok) break;
        tc_fence_after();
        // chunk k (0-3): head cc = 2*hh + k/2, columns 16*(k%2) .. +15 of that head; the
        // first 128 columns of the half are q (h = 0) or v (h = 1), the next 128 k or the gate
        const uint32_t tb = tmem + lane_off + h * 256 + hh * 64;
        uint32_t x0[2][16], x1[2][16];
        tmem_ld16(tb, x0[0]);
        tmem_ld16(tb + 128, x1[0]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int cur = k & 1;
          tmem_wait_ld_regs(x0[cur], x1[cur]);
          if (k + 1 < 4) {
            tmem_ld16(tb + (k + 1) * 16, x0[cur ^ 1]);
            tmem_ld16(tb + 128 + (k + 1) * 16, x1[cur ^ 1]);
          }
          if (!valid) continue;
          const int cc = 2 * hh + (k >> 1), c16 = (k & 1) * 16;
          uint32_t w0[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w0[e] = pack_f16x2_chk(__uint_as_float(x0[cur][2 * e]), __uint_as_float(x0[cur][2 * e + 1]), sat);
          __half* dst0 = (h == 0 ? q_out : v_out) + ((static_cast<size_t>(bi) * kHeads + cc) * N + j) * kHeadDim + c16;
          stg_v8(dst0, w0[0], w0[1], w0[2], w0[3], w0[4], w0[5], w0[6], w0[7]);
          uint32_t w1[8];
          if (h == 0) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              w1[e] = pack_f16x2_chk(__uint_as_float(x1[cur][2 * e]), __uint_as_float(x1[cur][2 * e + 1]), sat);
          } else {
            const float* bgc = bg_s + cc * 32 + c16;
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              const float4 g4 = *reinterpret_cast<const float4*>(bgc + e4 * 4);
              const float t0 = tanh_approx(__uint_as_float(x1[cur][e4 * 4 + 0]) + g4.x);
              const float t1 = tanh_approx(__uint_as_float(x1[cur][e4 * 4 + 1]) + g4.y);
              const float t2 = tanh_approx(__uint_as_float(x1[cur][e4 * 4 + 2]) + g4.z);
              const float t3 = tanh_approx(__uint_as_float(x1[cur][e4 * 4 + 3]) + g4.w);
              w1[2 * e4] = pack_f16x2(fmaf(0.5f, t0, 0.5f), fmaf(0.5f, t1, 0.5f));
              w1[2 * e4 + 1] = pack_f16x2(fmaf(0.5f, t2, 0.5f), fmaf(0.5f, t3, 0.5f));
            }
          }
          __half* dst1 = h == 0 ? k_out + ((static_cast<size_t>(bi) * kHeads + cc) * N + j) * kHeadDim + c16
                                : g_out + (static_cast<size_t>(bi) * N + j) * 128 + cc * 32 + c16;
          stg_v8(dst1, w1[0], w1[1], w1[2], w1[3], w1[4], w1[5], w1[6], w1[7]);
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
// K4: flash-style core. CTA = (query tile jt, head h, batch b, group of kR rows i).
//   warps 0-3   softmax warpgroup 0 (rows r = 0, 2), warps 4-7 warpgroup 1 (r = 1, 3);
//               thread = query row j of the tile; 224 registers each (setmaxnreg);
//   warp 8      producer: TMA for Q (once), K, V (4-stage ring) and the bias tile
//               (bf16, 2 stages, shared by the kR rows); all lanes stage the mask bias of each
//               step plus a flag telling whether the step has any masked / absent key;
//   warp 9      TMEM allocator + MMA issuer (lane 0); warps 10-11 only donate registers.
// Step t = kt * kR + r handles key tile kt of row r and uses S/P buffer t & 1, so each
// warpgroup owns one S and one P buffer and the two run concurrently. A warpgroup reads
// its whole S row slice into registers at once and frees the buffer, so the tensor core
// computes S(t+2) while the softmax of step t runs; the MMA issuer is a non-blocking
// state machine that issues S up to two steps ahead of P V.
// The softmax threads add the bf16 triangle bias row (widened by an integer shift) and, on
// flagged steps, the mask bias,
// take the max, exponentiate (base 2; q and the bias carry log2 e) and pack P. The tensor
// core only computes Q K^T and P V.
// TMEM columns: O_r at 32r (0-127), S at 128 + 128*sb, P (fp16 pairs) at 384 + 64*pb.
// The running max is raised lazily (only when a tile's max exceeds it by > 8, in log2
// units), so O is rescaled rarely; P then stays <= 2^8, well inside fp16.
// ----------------------------------------------------------------------------------
namespace k4 {
constexpr int kR = 4;
constexpr int kKVS = 4;
constexpr int kThreads = 384;
// Register split: the kernel is launched with 168 registers per thread (384 x 168 =
// 64512 per CTA); softmax warps raise to 224, warps 8-11 drop to 56: 256*224 + 128*56 = 64512.
constexpr int kLaunchRegs = 168, kSoftmaxRegs = 224, kOtherRegs = 56;
static_assert(256 * kSoftmaxRegs + 128 * kOtherRegs <= kThreads * kLaunchRegs, "register split");
constexpr uint32_t kQ = 0;
constexpr uint32_t kKV = 32768;
constexpr uint32_t kKVStage = 17408;  // K 8 KB | V 8 KB | mask bias 128 fp32 | flag
constexpr uint32_t kMB = 16384, kFlag = 16896;
constexpr uint32_t kBias = kKV + kKVS * kKVStage;  // bf16 bias tile [128 j][128 k] as 2 swizzled 64-key boxes
constexpr uint32_t kBiasStage = 32768;
constexpr uint32_t kBar = kBias + 2 * kBiasStage;
constexpr uint32_t kSmem = kBar + 256 + 1024;
static_assert(kSmem <= 232448, "K4 shared memory");
static_assert(kBias % 1024 == 0, "bias stage alignment");
constexpr float kLazy = 8.0f;
}  // namespace k4

struct K4Bars {
  uint64_t q_full;
  uint64_t kv_full[k4::kKVS];
  uint64_t kv_empty[k4::kKVS];
  uint64_t bias_full[2];
  uint64_t bias_empty[2];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t p_free[2];
  uint64_t o_ready[k4::kR];
  uint64_t o_final;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K4Bars) <= 256, "K4 barrier block");

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
  float2 d;
  asm("add.f32x2 %0, %1, %2;"
      : "=l"(reinterpret_cast<uint64_t&>(d))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
  return d;
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

__global__ void __launch_bounds__(k4::kThreads, 1)
    triatt_core_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                       const __grid_constant__ CUtensorMap v_map, const __grid_constant__ CUtensorMap bias_map,
                       const float* __restrict__ mask, int64_t mask_sb, int64_t mask_si, int64_t mask_sk,
                       float mask_scale, const __half* __restrict__ gate, __half* __restrict__ og, int N, int rows,
                       int n_igroups,
                       uint32_t* status) {
  using namespace k4;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  K4Bars* bars = reinterpret_cast<K4Bars*>(smem + kBar);
  CtaGuard* guard = &bars->guard;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int jt = blockIdx.x, h = blockIdx.y;
  const int b = blockIdx.z / n_igroups, ig = blockIdx.z % n_igroups;
  const int KT = (N + 127) / 128;
  const int T = KT * kR;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kKVS; ++s) {
      mbar_init(&bars->kv_full[s], 33);  // expect_tx arrival + 32 producer lanes after staging the mask bias
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->bias_full[x], 1);
      mbar_init(&bars->bias_empty[x], 256);  // both softmax warpgroups
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->s_free[x], 128);
      mbar_init(&bars->p_full[x], 128);
      mbar_init(&bars->p_free[x], 1);
    }
    for (int r = 0; r < kR; ++r) mbar_init(&bars->o_ready[r], 1);
    mbar_init(&bars->o_final, 1);
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;

  if (warp >= 8) {
    setmaxnreg_dec<kOtherRegs>();
    if (warp == 8) {
      // ------------------------------ producer ------------------------------
      int issued_kv = 0, issued_bias = 0;
      bool ok = true;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars->q_full, kR * 8192);
#pragma unroll
        for (int r = 0; r < kR; ++r) {
          const int i = min(ig * kR + r, rows - 1);
          tma_load_4d(smem + kQ + r * 8192, &q_map, &bars->q_full, 0, jt * 128, h, b * rows + i);
        }
      }
      for (int kt = 0; kt < KT && ok; ++kt) {
        const int bs = kt & 1;
        if (kt >= 2) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->bias_empty[bs], ((kt >> 1) - 1) & 1, guard, status,
                                                 kStatusTimeoutProducer));
          if (!ok) break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&bars->bias_full[bs], kBiasStage);
#pragma unroll
          for (int kh = 0; kh < 2; ++kh)
            tma_load_3d(smem + kBias + bs * kBiasStage + kh * 16384, &bias_map, &bars->bias_full[bs],
                        kt * 128 + kh * 64, jt * 128, b * kHeads + h);
        }
        ++issued_bias;
        for (int r = 0; r < kR; ++r) {
          const int t = kt * kR + r, s = t % kKVS;
          const int i = min(ig * kR + r, rows - 1);
          if (t >= kKVS) {
            ok = __all_sync(0xffffffffu, mbar_wait(&bars->kv_empty[s], ((t / kKVS) - 1) & 1, guard, status,
                                                   kStatusTimeoutProducer));
            if (!ok) break;
          }
          uint8_t* stage = smem + kKV + s * kKVStage;
          if (lane == 0) {
            mbar_arrive_expect_tx(&bars->kv_full[s], 16384);
            tma_load_4d(stage, &k_map, &bars->kv_full[s], 0, kt * 128, h, b * rows + i);
            tma_load_4d(stage + 8192, &v_map, &bars->kv_full[s], 0, kt * 128, h, b * rows + i);
          }
          float* mb = reinterpret_cast<float*>(stage + kMB);
          const float* mrow =
              mask ? mask + static_cast<int64_t>(b) * mask_sb + static_cast<int64_t>(i) * mask_si : nullptr;
          bool any = false;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int kk = kt * 128 + lane * 4 + e;
            float v;
            if (kk >= N) v = -INFINITY;
            else if (mrow) v = (mrow[static_cast<int64_t>(kk) * mask_sk] - 1.f) * mask_scale;
            else v = 0.f;
            mb[lane * 4 + e] = v;
            any |= (v != 0.f);
          }
          any = __any_sync(0xffffffffu, any);
          if (lane == 0) *reinterpret_cast<int*>(stage + kFlag) = any ? 1 : 0;
          mbar_arrive(&bars->kv_full[s]);
          ++issued_kv;
        }
      }
      if (!ok && lane == 0) {
        for (int t = (issued_kv > kKVS ? issued_kv - kKVS : 0); t < issued_kv; ++t)
          mbar_wait_drain(&bars->kv_full[t % kKVS], (t / kKVS) & 1);
        for (int kt = (issued_bias > 2 ? issued_bias - 2 : 0); kt < issued_bias; ++kt)
          mbar_wait_drain(&bars->bias_full[kt & 1], (kt >> 1) & 1);
        mbar_wait_drain(&bars->q_full, 0);
      }
    } else if (warp == 9 && lane == 0) {
      // ------------------------------ MMA issuer ------------------------------
      const uint32_t id_s = make_idesc_f16(128, 128, 0, 0);
      const uint32_t id_o = make_idesc_f16(128, 32, 0, 1);
      bool ok = mbar_wait(&bars->q_full, 0, guard, status, kStatusTimeoutMma);
      int ns = 0, npv = 0;  // next S step, next P V step
      uint64_t t0 = global_timer_ns();
      uint32_t spins = 0;
      while (ok && npv < T) {
        bool progress = false;
        // S(ns): needs its K stage and its S buffer freed by step ns-2
        if (ns < T && ns < npv + 2 + 1) {
          const int s = ns % kKVS, sb = ns & 1, r = ns % kR;
          if (mbar_test_wait(smem_u32(&bars->kv_full[s]), (ns / kKVS) & 1) &&
              (ns < 2 || mbar_test_wait(smem_u32(&bars->s_free[sb]), ((ns >> 1) - 1) & 1))) {
            tc_fence_after();
            const uint32_t qaddr = smem_u32(smem + kQ + r * 8192);
            const uint32_t kaddr = smem_u32(smem + kKV + s * kKVStage);
            const uint32_t dcol = tmem + 128 + sb * 128;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
              umma_ss(dcol, make_sdesc(qaddr + ks * 32, 16, 512, Swz::k64),
                      make_sdesc(kaddr + ks * 32, 16, 512, Swz::k64), id_s, ks > 0 ? 1u : 0u);
            umma_commit(&bars->s_full[sb]);
            ++ns;
            progress = true;
          }
        }
        // P V(npv): needs P written by the softmax of step npv
        if (npv < ns) {
          const int rp = npv % kR, kp = npv / kR, sp = npv % kKVS, pb = npv & 1;
          if (mbar_test_wait(smem_u32(&bars->p_full[pb]), (npv >> 1) & 1)) {
            tc_fence_after();
            const uint32_t vaddr = smem_u32(smem + kKV + sp * kKVStage + 8192);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              umma_ts(tmem + rp * 32, tmem + 384 + pb * 64 + ks * 8,
                      make_sdesc(vaddr + ks * 1024, 16, 512, Swz::k64), id_o, (kp > 0 || ks > 0) ? 1u : 0u);
            umma_commit(&bars->kv_empty[sp]);
            umma_commit(&bars->p_free[pb]);
            umma_commit(&bars->o_ready[rp]);
            ++npv;
            progress = true;
          }
        }
        if (progress) {
          t0 = global_timer_ns();
          spins = 0;
        } else if ((++spins & 63u) == 0) {
          if (guard->abort) {
            ok = false;
          } else if (global_timer_ns() - t0 > kWaitLimitNs) {
            guard->abort = 1;
            if (status) atomicOr(status, kStatusTimeoutMma);
            ok = false;
          }
        }
      }
      umma_commit(&bars->o_final);  // also drains whatever was issued before an abort
    }
  } else {
    // ------------------------------ softmax ------------------------------
    setmaxnreg_inc<kSoftmaxRegs>();
    const int wg = warp >> 2;  // 0 or 1: owns rows wg and wg + 2, S/P buffer wg
    const int quarter = warp & 3;
    const int jrow = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int sb = wg;
    const uint32_t scol = tmem + lane_off + 128 + sb * 128;
    float m_run0 = -INFINITY, m_run1 = -INFINITY, l_run0 = 0.f, l_run1 = 0.f;
    bool ok = true;
    for (int kt = 0; kt < KT && ok; ++kt) {
      const int bs = kt & 1;
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&bars->bias_full[bs], (kt >> 1) & 1, guard, status, kStatusTimeoutConsumer));
      if (!ok) break;
      const uint8_t* brow = smem + kBias + bs * kBiasStage;
      // not unrolled: one copy of the row step's long straight-line body keeps the
      // instruction footprint small
#pragma unroll 1
      for (int rr = 0; rr < 2; ++rr) {
        const int r = wg + 2 * rr;
        const int t = kt * kR + r, s = t % kKVS;
        bool w = mbar_wait(&bars->kv_full[s], (t / kKVS) & 1, guard, status, kStatusTimeoutConsumer);
        w = w && mbar_wait(&bars->s_full[sb], (t >> 1) & 1, guard, status, kStatusTimeoutConsumer);
        ok = __all_sync(0xffffffffu, w);
        if (!ok) break;
        tc_fence_after();
        uint32_t sv[128];
        tmem_ld32(scol + 0, *reinterpret_cast<uint32_t(*)[32]>(sv + 0));
        tmem_ld32(scol + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_ld32(scol + 64, *reinterpret_cast<uint32_t(*)[32]>(sv + 64));
        tmem_ld32(scol + 96, *reinterpret_cast<uint32_t(*)[32]>(sv + 96));
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars->s_free[sb]);  // the tensor core may now compute S(t + 2)

        // + triangle bias row j (bf16 -> fp32 by shifting into the high half)
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint4 bw = *reinterpret_cast<const uint4*>(brow + kh * 16384 + swz128(jrow, ch));
            const uint32_t wv[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int k = kh * 64 + ch * 8 + 2 * e;
              const float2 x = add_f32x2(make_float2(__uint_as_float(sv[k]), __uint_as_float(sv[k + 1])),
                                         make_float2(bf16_lo(wv[e]), bf16_hi(wv[e])));
              sv[k] = __float_as_uint(x.x);
              sv[k + 1] = __float_as_uint(x.y);
            }
          }
        const uint8_t* stage = smem + kKV + s * kKVStage;
        if (*reinterpret_cast<const volatile int*>(stage + kFlag)) {
          const float* mb = reinterpret_cast<const float*>(stage + kMB);
#pragma unroll
          for (int k4i = 0; k4i < 32; ++k4i) {
            const float4 m4 = *reinterpret_cast<const float4*>(mb + k4i * 4);
            sv[k4i * 4 + 0] = __float_as_uint(__uint_as_float(sv[k4i * 4 + 0]) + m4.x);
            sv[k4i * 4 + 1] = __float_as_uint(__uint_as_float(sv[k4i * 4 + 1]) + m4.y);
            sv[k4i * 4 + 2] = __float_as_uint(__uint_as_float(sv[k4i * 4 + 2]) + m4.z);
            sv[k4i * 4 + 3] = __float_as_uint(__uint_as_float(sv[k4i * 4 + 3]) + m4.w);
          }
        }
        // row max over four independent chains (a single chain serialises on the FMNMX latency)
        float mx4[4] = {__uint_as_float(sv[0]), __uint_as_float(sv[1]), __uint_as_float(sv[2]),
                        __uint_as_float(sv[3])};
#pragma unroll
        for (int k = 4; k < 124; k += 8)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            mx4[c] = max3f(mx4[c], __uint_as_float(sv[k + 2 * c]), __uint_as_float(sv[k + 2 * c + 1]));
        const float mx = max3f(max3f(mx4[0], mx4[1], __uint_as_float(sv[124])),
                               max3f(mx4[2], mx4[3], __uint_as_float(sv[125])),
                               fmaxf(__uint_as_float(sv[126]), __uint_as_float(sv[127])));
        const float m_old = rr == 0 ? m_run0 : m_run1;
        const float m_new = (mx > m_old + kLazy) ? mx : m_old;
        const float alpha = (m_new == m_old) ? 1.f : ex2f(m_old - m_new);
        const float2 negm = make_float2(-m_new, -m_new);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int k2 = 0; k2 < 64; ++k2) {
          float2 x = add_f32x2(make_float2(__uint_as_float(sv[2 * k2]), __uint_as_float(sv[2 * k2 + 1])), negm);
          x.x = ex2f(x.x);
          x.y = ex2f(x.y);
          acc[k2 & 3] = add_f32x2(acc[k2 & 3], x);  // four independent partial sums
          __half2 hp = __floats2half2_rn(x.x, x.y);
          sv[k2] = *reinterpret_cast<uint32_t*>(&hp);
        }
        const float2 a01 = add_f32x2(acc[0], acc[1]), a23 = add_f32x2(acc[2], acc[3]);
        const float sum = (a01.x + a23.x) + (a01.y + a23.y);
        if (rr == 0) {
          l_run0 = l_run0 * alpha + sum;
          m_run0 = m_new;
        } else {
          l_run1 = l_run1 * alpha + sum;
          m_run1 = m_new;
        }
        if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          // O_r must hold the sum through key tile kt-1 before it is rescaled.
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_ready[r], (kt - 1) & 1, guard, status,
                                                 kStatusTimeoutConsumer));
          if (!ok) break;
          tc_fence_after();
          uint32_t ov[32];
          tmem_ld32(tmem + lane_off + r * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(tmem + lane_off + r * 32, ov);
        }
        if (t >= 2) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->p_free[sb], ((t >> 1) - 1) & 1, guard, status,
                                                 kStatusTimeoutConsumer));
          if (!ok) break;
        }
        tc_fence_after();
        tmem_st32(tmem + lane_off + 384 + sb * 64, *reinterpret_cast<uint32_t(*)[32]>(sv + 0));
        tmem_st32(tmem + lane_off + 384 + sb * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->p_full[sb]);
      }
      if (ok) mbar_arrive(&bars->bias_empty[bs]);
    }
    // epilogue: O / l, times the gate, to og (rows wg and wg + 2). The gate rows are loaded
    // before waiting for the last P V, so their latency overlaps the drain.
    const int j = jt * 128 + jrow;
    uint4 gw[2][4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int i = ig * kR + wg + 2 * rr;
      const bool valid = ok && i < rows && j < N;
      const uint4* gp = reinterpret_cast<const uint4*>(gate + ((static_cast<size_t>(b) * rows + i) * N + j) * 128 +
                                                       h * kHeadDim);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) gw[rr][ch] = valid ? __ldg(gp + ch) : make_uint4(0u, 0u, 0u, 0u);
    }
    const bool fin = __all_sync(0xffffffffu, ok && mbar_wait(&bars->o_final, 0, guard, status,
                                                             kStatusTimeoutConsumer) && !guard->abort);
    if (fin) {
      uint32_t sat = 0;  // a gated output beyond the fp16 range was clamped
      tc_fence_after();
      uint32_t ov[2][32];
      tmem_ld32(tmem + lane_off + wg * 32, ov[0]);
      tmem_ld32(tmem + lane_off + (wg + 2) * 32, ov[1]);
      tmem_wait_ld();
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int i = ig * kR + wg + 2 * rr;
        if (i < rows && j < N) {
          const float inv = 1.f / (rr == 0 ? l_run0 : l_run1);
          const size_t pair = (static_cast<size_t>(b) * rows + i) * N + j;
          uint32_t o16[16];
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const __half2* gh = reinterpret_cast<const __half2*>(&gw[rr][ch]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 gf = __half22float2(gh[e]);
              o16[ch * 4 + e] = pack_f16x2_chk(__uint_as_float(ov[rr][ch * 8 + 2 * e]) * inv * gf.x,
                                               __uint_as_float(ov[rr][ch * 8 + 2 * e + 1]) * inv * gf.y, sat);
            }
          }
          __half* op = og + pair * 128 + h * kHeadDim;  // 64 contiguous bytes, 64-byte aligned
          stg_v8(op, o16[0], o16[1], o16[2], o16[3], o16[4], o16[5], o16[6], o16[7]);
          stg_v8(op + 16, o16[8], o16[9], o16[10], o16[11], o16[12], o16[13], o16[14], o16[15]);
        }
      }
      flag_saturation(sat, status);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------------
// K4e: persistent update = og W_o^T + b_o (+ residual), written through the (possibly
// transposed) pair descriptor. Tile = 128 pairs of row i of the problem; each tile is
// handled as four 32-channel fp32 slabs [128 pairs][32] that travel through a ring of
// four shared-memory buffers: the producer TMA-loads the residual slab of z into a
// buffer, the epilogue adds the accumulator and bias in place, and a TMA store writes it
// out, so every global access is a bulk tensor copy. 192 threads:
//   warps 0-3  epilogue: thread = pair (TMEM lane);
//   warp 4     lane 0: TMA producer (W_o once, og tiles double buffered, z slabs);
//   warp 5     lane 0: MMA issuer (TMEM double buffered, 128 columns per tile).
// Shared memory: W4 32 KB | og 2 x 32 KB | slabs 4 x 16 KB | b_o | barriers.
// ----------------------------------------------------------------------------------
namespace k4e {
constexpr int kThreads = 192;
constexpr int kSlabs = 4;
constexpr uint32_t kW = 0, kA = 32768, kO = 98304, kVec = 98304 + kSlabs * 16384, kBar = kVec + 512;
constexpr uint32_t kSmem = kBar + 256 + 1024;
static_assert(kSmem <= 232448, "K4e shared memory");
}  // namespace k4e

struct K4eBars {
  uint64_t wbar;
  uint64_t a_full[2], a_empty[2];
  uint64_t d_full[2], d_empty[2];
  uint64_t o_full[k4e::kSlabs], o_empty[k4e::kSlabs];
  uint64_t slab_ready[k4e::kSlabs];  // 128 epilogue threads wrote the slab
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K4eBars) <= 256, "K4e barrier block");

// Destinations of the peer form of K4e: the pair-grid transpose of a row shard, straight into
// the P ranks' shards. Tile (b, i, j0..j0+127) goes to rank q = j0 / R as its pairs
// (b, j - q*R, row0 + i): map[q] addresses rank q's shard [B][R][N][128] as (channel, row,
// column, b) with a box of 32 channels x 128 rows, so the tile's slabs are TMA stores into
// the peer's memory over NVLink (plain stores, no multicast).
constexpr int kMaxPeers = 8;
struct K4ePeers {
  CUtensorMap map[kMaxPeers];
  int R, row0;
};

// kDrop: the update is multiplied by the channel dropout `drop` before the residual add
// (out = z + keep * scale * update); the plain instantiation ignores `drop`.
// kPeer: the finished tile goes to the peers' transposed shards (K4ePeers), not to out_map.
template <bool kDrop, bool kPeer>
__global__ void __launch_bounds__(k4e::kThreads, 1)
    triatt_finish_kernel(const __grid_constant__ CUtensorMap og_map, const __grid_constant__ CUtensorMap w_map,
                         const __grid_constant__ CUtensorMap z_map, const __grid_constant__ CUtensorMap out_map,
                         const float* __restrict__ vec, int N, int rows, int add_residual, int n_jt,
                         int n_tiles, uint32_t* status, const DropArgs drop, const __grid_constant__ K4ePeers peers) {
  using namespace k4e;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  K4eBars* bars = reinterpret_cast<K4eBars*>(smem + kBar);
  CtaGuard* guard = &bars->guard;
  float* sbo = reinterpret_cast<float*>(smem + kVec);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(&bars->wbar, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->a_full[x], 1);
      mbar_init(&bars->a_empty[x], 1);
      mbar_init(&bars->d_full[x], 1);
      mbar_init(&bars->d_empty[x], 128);
    }
    for (int x = 0; x < kSlabs; ++x) {
      mbar_init(&bars->o_full[x], 1);
      mbar_init(&bars->o_empty[x], 1);
      mbar_init(&bars->slab_ready[x], 128);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (tid < 128) sbo[tid] = vec[tapack::kVBo + tid];
  if (warp == 5) {
    tmem_alloc(&bars->tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;

  if (warp == 4) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->wbar, 32768);
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) tma_load_2d(smem + kW + kh * 16384, &w_map, &bars->wbar, kh * 64, 0);
      bool ok = true;
      int it = 0, issued_a = 0, slab = 0;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        const int jt = tile % n_jt, bi = tile / n_jt;
        const int i = bi % rows, b = bi / rows, j0 = jt * 128;
        if (it >= 2 && !mbar_wait(&bars->a_empty[s], ((it >> 1) - 1) & 1, guard, status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->a_full[s], 32768);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
          tma_load_3d(smem + kA + s * 32768 + kh * 16384, &og_map, &bars->a_full[s], kh * 64, jt * 128, bi);
        ++issued_a;
        for (int cc = 0; cc < 4; ++cc, ++slab) {
          const int sl = slab % kSlabs;
          if (slab >= kSlabs && !mbar_wait(&bars->o_empty[sl], ((slab / kSlabs) - 1) & 1, guard, status,
                                           kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          if (add_residual) {
            mbar_arrive_expect_tx(&bars->o_full[sl], 16384);
            tma_load_4d(smem + kO + sl * 16384, &z_map, &bars->o_full[sl], cc * 32, j0, i, b);
          } else {
            mbar_arrive(&bars->o_full[sl]);
          }
        }
      }
      if (!ok) {
        for (int t = (issued_a > 2 ? issued_a - 2 : 0); t < issued_a; ++t)
          mbar_wait_drain(&bars->a_full[t & 1], (t >> 1) & 1);
        for (int t = (slab > kSlabs ? slab - kSlabs : 0); t < slab; ++t)
          mbar_wait_drain(&bars->o_full[t % kSlabs], (t / kSlabs) & 1);
      }
      mbar_wait_drain(&bars->wbar, 0);
    }
  } else if (warp == 5) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(&bars->wbar, 0, guard, status, kStatusTimeoutMma);
      const uint32_t idesc = make_idesc_f16(128, 128, 0, 0);
      const uint32_t w0 = smem_u32(smem + kW);
      int it = 0;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        ok = mbar_wait(&bars->a_full[s], (it >> 1) & 1, guard, status, kStatusTimeoutMma);
        if (ok && it >= 2) ok = mbar_wait(&bars->d_empty[s], ((it >> 1) - 1) & 1, guard, status, kStatusTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + kA + s * 32768);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int kh = ks >> 2, kin = ks & 3;
          umma_ss(tmem + s * 128, make_sdesc(a0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128),
                  make_sdesc(w0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128), idesc, ks > 0 ? 1u : 0u);
        }
        umma_commit(&bars->d_full[s]);
        umma_commit(&bars->a_empty[s]);
      }
      if (!ok) {
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else {
    // ------------------------- epilogue: thread = pair -------------------------
    const int p = tid;  // warps 0-3
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const bool issuer = (tid == 0);
    int it = 0, slab = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      const int jt = tile % n_jt, bi = tile / n_jt;
      const int i = bi % rows, b = bi / rows, j0 = jt * 128;
      uint4 keep = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (kDrop) keep = drop_keep(drop, b, i, j0 + p, N);  // latency hidden under the wait
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
        const uint32_t kw = kDrop ? drop_word(keep, cc) : 0u;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int n = cc * 32 + q * 4;
          float4 o = make_float4(__uint_as_float(d[q * 4 + 0]) + sbo[n + 0], __uint_as_float(d[q * 4 + 1]) + sbo[n + 1],
                                 __uint_as_float(d[q * 4 + 2]) + sbo[n + 2], __uint_as_float(d[q * 4 + 3]) + sbo[n + 3]);
          if constexpr (kDrop) {
            const float sc = drop.scale;
            o.x *= ((kw >> (q * 4 + 0)) & 1u) ? sc : 0.f;
            o.y *= ((kw >> (q * 4 + 1)) & 1u) ? sc : 0.f;
            o.z *= ((kw >> (q * 4 + 2)) & 1u) ? sc : 0.f;
            o.w *= ((kw >> (q * 4 + 3)) & 1u) ? sc : 0.f;
          }
          if (add_residual) {
            const float4 zv = lds_f4(ob + swz128(p, q));
            o.x += zv.x;
            o.y += zv.y;
            o.z += zv.z;
            o.w += zv.w;
          }
          *reinterpret_cast<float4*>(ob + swz128(p, q)) = o;
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->slab_ready[sl]);
        if (warp == 0) {
          // one thread stores the slab once all 128 have written it (a bounded wait, so
          // that an abort elsewhere cannot leave threads parked at a barrier)
          bool iok = true;
          if (issuer) {
            iok = mbar_wait(&bars->slab_ready[sl], (slab / kSlabs) & 1, guard, status, kStatusTimeoutConsumer);
            if (iok) {
              if constexpr (kPeer) {
                const int q = j0 / peers.R;
                tma_store_4d(&peers.map[q], ob, cc * 32, j0 - q * peers.R, peers.row0 + i, b);
              } else {
                tma_store_4d(&out_map, ob, cc * 32, j0, i, b);
              }
              tma_store_commit();
              // a slab buffer is free again once its store has read it; keep two stores in flight
              tma_store_wait_read_le1();
              if (slab >= 1) mbar_arrive(&bars->o_empty[(slab - 1) % kSlabs]);
            }
          }
          ok = __shfl_sync(0xffffffffu, iok ? 1 : 0, 0) != 0;
        }
        if (!ok) break;
      }
      tc_fence_before();
      mbar_arrive(&bars->d_empty[s]);
    }
    if (issuer) {
      tma_store_wait_all();
      if (ok && slab >= 1) mbar_arrive(&bars->o_empty[(slab - 1) % kSlabs]);
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
struct TriattWs {
  size_t q, k, v, g, og, bias, total;
};

// q, k, v, g, og cover the `rows` local problem rows; the bias always covers all N rows
// (the attention core reads every row j of it).
static TriattWs triatt_layout(int64_t B, int64_t rows, int64_t N) {
  TriattWs w;
  const size_t pair16 = round_up(static_cast<size_t>(B) * rows * N * 128 * 2, 256);
  const size_t bias = round_up(static_cast<size_t>(N) * B * kHeads * round_up(N, 8) * 2, 256);
  w.q = 0;
  w.k = w.q + pair16;
  w.v = w.k + pair16;
  w.g = w.v + pair16;
  w.og = w.g + pair16;
  w.bias = w.og + pair16;
  w.total = w.bias + bias;
  return w;
}

// q / k / v: [B*rows(i)][H][N(j)][32] fp16, box (32, 128, 1, 1), 64-B swizzle.
static int make_head_map(CUtensorMap* m, const void* base, int64_t BR, int64_t N) {
  uint64_t dims[4] = {32, static_cast<uint64_t>(N), static_cast<uint64_t>(kHeads), static_cast<uint64_t>(BR)};
  uint64_t strides[3] = {64, static_cast<uint64_t>(N) * 64, static_cast<uint64_t>(N) * 64 * kHeads};
  uint32_t box[4] = {32, 128, 1, 1};
  return encode_tmap(m, TmaType::kF16, 4, base, dims, strides, box, 64);
}

// g / og: [B*rows(i)][N(j)][128] fp16, box (64, 128, 1), 128-B swizzle.
static int make_hidden_map(CUtensorMap* m, const void* base, int64_t BR, int64_t N) {
  uint64_t dims[3] = {128, static_cast<uint64_t>(N), static_cast<uint64_t>(BR)};
  uint64_t strides[2] = {256, static_cast<uint64_t>(N) * 256};
  uint32_t box[3] = {64, 128, 1};
  return encode_tmap(m, TmaType::kF16, 3, base, dims, strides, box, 128);
}

// bias: [N(j)][B*H][ldn] bf16, addressed as (k, j, b*H + h); box (64 k, 128 j, 1), 128-B swizzle.
static int make_bias_map(CUtensorMap* m, const void* base, int64_t B, int64_t N) {
  const uint64_t ldn = round_up(static_cast<uint64_t>(N), 8);
  const uint64_t BH = static_cast<uint64_t>(B) * kHeads;
  uint64_t dims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(N), BH};
  uint64_t strides[2] = {ldn * 2 * BH, ldn * 2};
  uint32_t box[3] = {64, 128, 1};
  return encode_tmap(m, TmaType::kBF16, 3, base, dims, strides, box, 128);
}

// Row-shard arguments shared by the stage entry points: `rows` local problem rows starting
// at global row `row0` (all of them, rows = N and row0 = 0, when unsharded).
static int rows_check(const char* who, int starting, int64_t B, int64_t rows, int64_t N, int64_t row0) {
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535) || !dims_ok(rows, 65535) || row0 < 0 || row0 + rows > N)
    return fail(GTK_ERR_INVALID_ARG, std::string(who) + ": bad B/rows/N/row0");
  if (!starting && (rows != N || row0 != 0))
    return fail(GTK_ERR_UNSUPPORTED, std::string(who) + ": the ending orientation runs on whole (unsharded) pair "
                                                         "tensors; a row-sharded caller transposes the shards and "
                                                         "runs the starting orientation");
  return GTK_OK;
}

static int triatt_check(int c_in, int c_hidden, int heads) {
  if (c_in != 128 || heads != kHeads || c_hidden % kHeads || c_hidden < kHeads || c_hidden > 128)
    return fail(GTK_ERR_UNSUPPORTED, "triatt: the tuned kernels take c_in = 128 with 4 heads of head_dim <= 32");
  return GTK_OK;
}

}  // namespace gtk

using namespace gtk;

extern "C" {

// The tuned kernels: c_in = 128 and 4 heads of head_dim <= 32 (the 4 x 32 of the benchmark,
// and, with the heads zero-padded to 32 in the packed weights, the reference's default
// c_hidden_tri_att = 32 with 4 heads and any other 4 x d).
static bool triatt_tuned(int c_in, int c_hidden, int heads) {
  return c_in == 128 && heads == kHeads && c_hidden % kHeads == 0 && c_hidden >= kHeads && c_hidden <= 128;
}

size_t gtk_triatt_packed_bytes(int c_in, int c_hidden, int heads) {
  if (!triatt_tuned(c_in, c_hidden, heads)) return gen::triatt_packed_bytes(c_in, c_hidden, heads);
  return tapack::kBytes;
}

int gtk_triatt_pack(const gtk_triatt_params* params, int c_in, int c_hidden, int heads, void* packed,
                    size_t packed_bytes, void* stream) {
  if (!triatt_tuned(c_in, c_hidden, heads))
    return gen::triatt_pack(params, c_in, c_hidden, heads, packed, packed_bytes, stream);
  if (int e = triatt_check(c_in, c_hidden, heads)) return e;
  if (!params) return fail(GTK_ERR_INVALID_ARG, "params is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < tapack::kBytes) return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  const float* const* pp = reinterpret_cast<const float* const*>(params);
  for (int i = 0; i < 10; ++i)
    if (!pp[i]) return fail(GTK_ERR_INVALID_ARG, "a triatt parameter pointer is NULL");
  if (int e = check_device()) return e;
  const int d = c_hidden / heads;
  const float q_scale = kLog2e / std::sqrt(static_cast<float>(d));
  triatt_pack_kernel<<<64, 256, 0, static_cast<cudaStream_t>(stream)>>>(*params, static_cast<uint8_t*>(packed),
                                                                         q_scale, d);
  return check_launch("triatt_pack_kernel");
}

size_t gtk_triatt_workspace_bytes(int64_t B, int64_t N, int c_in, int c_hidden, int heads) {
  if (!triatt_tuned(c_in, c_hidden, heads)) return gen::triatt_workspace_bytes(B, N, c_in, c_hidden, heads);
  if (B < 1 || N < 1) return 0;
  return triatt_layout(B, N, N).total;
}

int gtk_triatt_workspace_offsets(int64_t B, int64_t rows, int64_t N, int64_t* offsets) {
  if (!offsets || B < 1 || N < 1 || rows < 1 || rows > N)
    return fail(GTK_ERR_INVALID_ARG, "triatt_workspace_offsets: bad arguments");
  const TriattWs w = triatt_layout(B, rows, N);
  offsets[0] = static_cast<int64_t>(w.q);
  offsets[1] = static_cast<int64_t>(w.k);
  offsets[2] = static_cast<int64_t>(w.v);
  offsets[3] = static_cast<int64_t>(w.g);
  offsets[4] = static_cast<int64_t>(w.og);
  offsets[5] = static_cast<int64_t>(w.bias);
  offsets[6] = static_cast<int64_t>(w.total);
  return GTK_OK;
}

int gtk_triatt_project(int starting, const float* z, const void* packed, void* workspace, int64_t B, int64_t rows,
                       int64_t N, int64_t row0, uint32_t* status, void* stream) {
  if (int e = rows_check("triatt_project", starting, B, rows, N, row0)) return e;
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  if (int e = check_device()) return e;
  const TriattWs w = triatt_layout(B, rows, N);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  const int64_t n_jt = (N + 127) / 128;
  const int64_t n_tiles = B * rows * n_jt;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "triatt_project: too many tiles");
  CUtensorMap wm, zm;
  if (int e = make_weight_map(&wm, pk + tapack::kW3, 512, 128)) return e;
  if (int e = make_pair_map(&zm, z, B, rows, N, !starting)) return e;
  if (int e = ensure_smem(reinterpret_cast<const void*>(triatt_project_kernel), k3::kSmem)) return e;
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  triatt_project_kernel<<<grid, k3::kThreads, k3::kSmem, static_cast<cudaStream_t>(stream)>>>(
      wm, zm, reinterpret_cast<const float*>(pk + tapack::kVec), reinterpret_cast<__half*>(ws + w.q),
      reinterpret_cast<__half*>(ws + w.k), reinterpret_cast<__half*>(ws + w.v), reinterpret_cast<__half*>(ws + w.g),
      reinterpret_cast<__nv_bfloat16*>(ws + w.bias), static_cast<int>(N), static_cast<int>(rows),
      static_cast<int>(B), static_cast<int>(row0), static_cast<int>(round_up(N, 8)), static_cast<int>(n_jt),
      static_cast<int>(n_tiles), status);
  return check_launch("triatt_project_kernel");
}

int gtk_triatt_core(int starting, const float* mask, void* workspace, int64_t B, int64_t rows, int64_t N,
                    int64_t row0, float inf, uint32_t* status, void* stream) {
  if (int e = rows_check("triatt_core", starting, B, rows, N, row0)) return e;
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (int e = check_device()) return e;
  const TriattWs w = triatt_layout(B, rows, N);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  CUtensorMap qm, km, vm, bm;
  if (int e = make_head_map(&qm, ws + w.q, B * rows, N)) return e;
  if (int e = make_head_map(&km, ws + w.k, B * rows, N)) return e;
  if (int e = make_head_map(&vm, ws + w.v, B * rows, N)) return e;
  if (int e = make_bias_map(&bm, ws + w.bias, B, N)) return e;
  if (int e = ensure_smem(reinterpret_cast<const void*>(triatt_core_kernel), k4::kSmem)) return e;
  {
    // The kernel redistributes registers between warp roles (setmaxnreg); that is only safe
    // when it is launched with exactly the per-thread count the split was computed for.
    static int regs = -1;
    if (regs < 0) {
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(triatt_core_kernel)) != cudaSuccess)
        return fail(GTK_ERR_CUDA, "cudaFuncGetAttributes(triatt_core_kernel) failed");
      regs = fa.numRegs;
    }
    if (regs != k4::kLaunchRegs)
      return fail(GTK_ERR_CUDA, "triatt_core_kernel built with " + std::to_string(regs) +
                                    " registers/thread; its register split needs " +
                                    std::to_string(k4::kLaunchRegs));
  }
  const int n_ig = static_cast<int>((rows + k4::kR - 1) / k4::kR);
  if (static_cast<int64_t>(B) * n_ig > 65535) return fail(GTK_ERR_INVALID_ARG, "triatt_core: grid too large");
  dim3 grid(static_cast<unsigned>((N + 127) / 128), kHeads, static_cast<unsigned>(B * n_ig));
  // the mask is the whole problem's [B][N][N]; a shard's rows start at row row0
  const int64_t si = starting ? N : 1, sk = starting ? 1 : N;
  const float* mrow0 = mask ? mask + row0 * si : nullptr;
  triatt_core_kernel<<<grid, k4::kThreads, k4::kSmem, static_cast<cudaStream_t>(stream)>>>(
      qm, km, vm, bm, mrow0, N * N, si, sk, inf * kLog2e, reinterpret_cast<const __half*>(ws + w.g),
      reinterpret_cast<__half*>(ws + w.og), static_cast<int>(N), static_cast<int>(rows), n_ig, status);
  return check_launch("triatt_core_kernel");
}

}  // extern "C"

namespace gtk {

// K4e launch; `drop` with a NULL keep array selects the plain instantiation.
static int triatt_finish_launch(int starting, const float* z, const void* packed, void* workspace, float* out,
                                int add_residual, int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream,
                                const DropArgs& drop) {
  if (int e = rows_check("triatt_finish", starting, B, rows, N, 0)) return e;
  if (int e = check_ptr(out, "out")) return e;
  if (add_residual)
    if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  if (int e = check_device()) return e;
  const TriattWs w = triatt_layout(B, rows, N);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  const int64_t n_jt = (N + 127) / 128;
  const int64_t n_tiles = B * rows * n_jt;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "triatt_finish: too many tiles");
  CUtensorMap am, wm, zm, om;
  if (int e = make_hidden_map(&am, ws + w.og, B * rows, N)) return e;
  if (int e = make_weight_map(&wm, pk + tapack::kW4, 128, 128)) return e;
  if (int e = make_pair_map(&zm, add_residual ? z : out, B, rows, N, !starting)) return e;
  if (int e = make_pair_map(&om, out, B, rows, N, !starting)) return e;
  const bool dropping = drop.keep != nullptr;
  const void* kern = dropping ? reinterpret_cast<const void*>(triatt_finish_kernel<true, false>)
                              : reinterpret_cast<const void*>(triatt_finish_kernel<false, false>);
  if (int e = ensure_smem(kern, k4e::kSmem)) return e;
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  const float* vec = reinterpret_cast<const float*>(pk + tapack::kVec);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const K4ePeers none{};
  if (dropping)
    triatt_finish_kernel<true, false><<<grid, k4e::kThreads, k4e::kSmem, st>>>(
        am, wm, zm, om, vec, static_cast<int>(N), static_cast<int>(rows), add_residual, static_cast<int>(n_jt),
        static_cast<int>(n_tiles), status, drop, none);
  else
    triatt_finish_kernel<false, false><<<grid, k4e::kThreads, k4e::kSmem, st>>>(
        am, wm, zm, om, vec, static_cast<int>(N), static_cast<int>(rows), add_residual, static_cast<int>(n_jt),
        static_cast<int>(n_tiles), status, drop, none);
  return check_launch("triatt_finish_kernel");
}

// Rank q's shard [B][R][N][128] fp32 addressed as (channel, row, column, b), box 32 x 128 rows.
static int make_shard_rows_map(CUtensorMap* m, const void* base, int64_t B, int64_t R, int64_t N) {
  const uint64_t row = 128 * 4;
  uint64_t dims[4] = {128, static_cast<uint64_t>(R), static_cast<uint64_t>(N), static_cast<uint64_t>(B)};
  uint64_t strides[3] = {row * N, row, row * N * R};
  uint32_t box[4] = {32, 128, 1, 1};
  return encode_tmap(m, TmaType::kF32, 4, base, dims, strides, box, 128);
}

static int triatt_forward_impl(int starting, const float* z, const float* mask, const void* packed, float* out,
                               int add_residual, const DropArgs& drop, void* workspace, size_t workspace_bytes,
                               int64_t B, int64_t N, int c_in, int c_hidden, int heads, float inf, uint32_t* status,
                               void* stream) {
  if (!triatt_tuned(c_in, c_hidden, heads))  // every other shape: the general path
    return gen::triatt_forward(starting, z, mask, packed, out, add_residual, drop, workspace, workspace_bytes, B, N,
                               c_in, c_hidden, heads, inf, status, stream);
  if (int e = triatt_check(c_in, c_hidden, heads)) return e;
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535)) return fail(GTK_ERR_INVALID_ARG, "triatt: bad B/N");
  if (workspace_bytes < triatt_layout(B, N, N).total) return fail(GTK_ERR_WORKSPACE, "triatt: workspace too small");
  if (int e = gtk_triatt_project(starting, z, packed, workspace, B, N, N, 0, status, stream)) return e;
  if (int e = gtk_triatt_core(starting, mask, workspace, B, N, N, 0, inf, status, stream)) return e;
  return triatt_finish_launch(starting, z, packed, workspace, out, add_residual, B, N, N, status, stream, drop);
}

}  // namespace gtk

extern "C" {

int gtk_triatt_finish(int starting, const float* z, const void* packed, void* workspace, float* out, int add_residual,
                      int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream) {
  return triatt_finish_launch(starting, z, packed, workspace, out, add_residual, B, rows, N, status, stream,
                              DropArgs{});
}

int gtk_triatt_finish_to_peers(const float* z, const void* packed, void* workspace, const uint64_t* dst_bases, int P,
                               int64_t B, int64_t rows, int64_t N, int64_t row0, int add_residual, uint32_t* status,
                               void* stream) {
  if (P < 1 || P > kMaxPeers || !dst_bases) return fail(GTK_ERR_INVALID_ARG, "triatt_finish_to_peers: bad P");
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535) || rows < 1 || rows * P != N || row0 < 0 || row0 % rows ||
      row0 + rows > N)
    return fail(GTK_ERR_INVALID_ARG, "triatt_finish_to_peers: rows * P must equal N, row0 a multiple of rows");
  if (rows % 128) return fail(GTK_ERR_UNSUPPORTED, "triatt_finish_to_peers: rows per rank must be a multiple of 128");
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_ptr(workspace, "workspace", 256)) return e;
  for (int q = 0; q < P; ++q)
    if (int e = check_ptr(reinterpret_cast<const void*>(dst_bases[q]), "peer shard")) return e;
  if (int e = check_device()) return e;
  const TriattWs w = triatt_layout(B, rows, N);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  const int64_t n_jt = N / 128;
  const int64_t n_tiles = B * rows * n_jt;
  CUtensorMap am, wm, zm;
  if (int e = make_hidden_map(&am, ws + w.og, B * rows, N)) return e;
  if (int e = make_weight_map(&wm, pk + tapack::kW4, 128, 128)) return e;
  if (int e = make_pair_map(&zm, z, B, rows, N, false)) return e;
  K4ePeers peers{};
  peers.R = static_cast<int>(rows);
  peers.row0 = static_cast<int>(row0);
  for (int q = 0; q < P; ++q)
    if (int e = make_shard_rows_map(&peers.map[q], reinterpret_cast<const void*>(dst_bases[q]), B, rows, N)) return e;
  const void* kern = reinterpret_cast<const void*>(triatt_finish_kernel<false, true>);
  if (int e = ensure_smem(kern, k4e::kSmem)) return e;
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  const float* vec = reinterpret_cast<const float*>(pk + tapack::kVec);
  triatt_finish_kernel<false, true><<<grid, k4e::kThreads, k4e::kSmem, static_cast<cudaStream_t>(stream)>>>(
      am, wm, zm, zm, vec, static_cast<int>(N), static_cast<int>(rows), add_residual, static_cast<int>(n_jt),
      static_cast<int>(n_tiles), status, DropArgs{}, peers);
  return check_launch("triatt_finish_kernel (to peers)");
}

int gtk_triatt_forward(int starting, const float* z, const float* mask, const void* packed, float* out,
                       int add_residual, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_in,
                       int c_hidden, int heads, float inf, uint32_t* status, void* stream) {
  return triatt_forward_impl(starting, z, mask, packed, out, add_residual, DropArgs{}, workspace, workspace_bytes, B,
                             N, c_in, c_hidden, heads, inf, status, stream);
}

int gtk_triatt_forward_dropout(int starting, const float* z, const float* mask, const void* packed, float* out,
                               int add_residual, const gtk_dropout* dropout, void* workspace, size_t workspace_bytes,
                               int64_t B, int64_t N, int c_in, int c_hidden, int heads, float inf, uint32_t* status,
                               void* stream) {
  DropArgs d{};
  // K4e works in the problem's frame, which is z^T for the ending node.
  if (int e = drop_args(dropout, B, N, /*transposed=*/!starting, c_in, &d)) return e;
  return triatt_forward_impl(starting, z, mask, packed, out, add_residual, d, workspace, workspace_bytes, B, N, c_in,
                             c_hidden, heads, inf, status, stream);
}

}  // extern "C"
