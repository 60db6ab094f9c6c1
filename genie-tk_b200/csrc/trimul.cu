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

#include <mutex>
#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"
#include "general.h"

namespace gtk {

// ----------------------------------------------------------------------------------
// Packed weights (built by trimul_pack_kernel from the fp32 module parameters).
// All 16-bit operands are fp16 (tcgen05 kind::f16, fp32 accumulate): each is bounded --
// LayerNorm outputs, fan-in-scaled weights, gated projections, the 1/K-scaled contraction --
// and fp16 keeps 3 more mantissa bits than bf16 at the same tensor-core rate. Conversions
// saturate to the finite fp16 range.
//   W1  fp16 [512][128]: rows 0-127 linear_a_p, 128-255 linear_a_g / 2, 256-383 linear_b_p,
//                        384-511 linear_b_g / 2, each times gamma_in (nn.Linear [out, in] =
//                        K-major B operand; the gates' 1/2 feeds sigmoid(x) = (1 + tanh(x/2))/2)
//   W2  fp16 [256][128]: rows 0-127 linear_g * gamma_in / 2, 128-255 linear_z * gamma_out
//   vec fp32: b1[512] = the four projection biases + W beta_in (gate entries halved too),
//             b_g[128] = (b_g + W_g beta_in) / 2,
//             u[128] = sum_c W2[128+n][c] (fp16-rounded), v[128] = linear_z(beta_out) + b_z.
// Both LayerNorm affines are folded into the weights: LN(x) W^T + b = xhat (W*gamma)^T +
// (W beta + b) with xhat = (x - mu) * rstd, so the kernels' LayerNorm producers write xhat
// alone; for LN_out the mean term is folded too:
// LN_out(x) W_z^T + b_z = rstd * (x (W_z*gamma)^T - mu * u) + v for per-pair mean mu, rstd.
// ----------------------------------------------------------------------------------
namespace tmpack {
constexpr size_t kW1 = 0;
constexpr size_t kW2 = 512 * 128 * 2;
constexpr size_t kVec = kW2 + 256 * 128 * 2;
constexpr int kVB1 = 0, kVBg = 512, kVU = 640, kVV = 768, kVC = 896, kVecFloats = 900;  // kVC: real c_hidden
constexpr size_t kBytes = kVec + kVecFloats * 4;
}  // namespace tmpack

// Packs a multiplicative update of c_hidden = c <= 128 (c_z = 128) into the tuned 128-channel
// layout: hidden channels past c have zero projection rows and biases, so their a / b planes,
// and with them their x planes, are exactly zero; W_z gets zero columns there, and K2e takes
// LN_out's statistics over the c real channels (kVC).
__global__ void trimul_pack_kernel(gtk_trimul_params p, uint8_t* packed, int c) {
  __half* w1 = reinterpret_cast<__half*>(packed + tmpack::kW1);
  __half* w2 = reinterpret_cast<__half*>(packed + tmpack::kW2);
  float* vec = reinterpret_cast<float*>(packed + tmpack::kVec);
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int nthreads = gridDim.x * blockDim.x;
  for (int e = tid; e < 512 * 128; e += nthreads) {
    const int r = e >> 7, col = e & 127, h = r & 127;
    const float* src = r < 128 ? p.a_p_w : r < 256 ? p.a_g_w : r < 384 ? p.b_p_w : p.b_g_w;
    w1[e] = f16_sat(h < c ? src[h * 128 + col] * p.ln_in_w[col] * (((r >> 7) & 1) ? 0.5f : 1.f) : 0.f);
  }
  for (int e = tid; e < 256 * 128; e += nthreads) {
    const int r = e >> 7, col = e & 127;
    float val;
    if (r < 128) val = 0.5f * p.g_w[r * 128 + col] * p.ln_in_w[col];
    else val = col < c ? p.z_w[(r - 128) * c + col] * p.ln_out_w[col] : 0.f;
    w2[e] = f16_sat(val);
  }
  for (int e = tid; e < 512; e += nthreads) {
    const int r = e & 127;
    const float* w = e < 128 ? p.a_p_w : e < 256 ? p.a_g_w : e < 384 ? p.b_p_w : p.b_g_w;
    const float* bb = e < 128 ? p.a_p_b : e < 256 ? p.a_g_b : e < 384 ? p.b_p_b : p.b_g_b;
    float acc = 0.f;
    if (r < c) {
      acc = bb[r];
      for (int col = 0; col < 128; ++col) acc += w[r * 128 + col] * p.ln_in_b[col];
    }
    vec[tmpack::kVB1 + e] = acc * (((e >> 7) & 1) ? 0.5f : 1.f);
  }
  for (int e = tid; e < 128; e += nthreads) {
    float bg = p.g_b[e];
    for (int col = 0; col < 128; ++col) bg += p.g_w[e * 128 + col] * p.ln_in_b[col];
    vec[tmpack::kVBg + e] = 0.5f * bg;
    float u = 0.f, v = p.z_b[e];
    for (int col = 0; col < c; ++col) {
      u += __half2float(f16_sat(p.z_w[e * c + col] * p.ln_out_w[col]));
      v += p.z_w[e * c + col] * p.ln_out_b[col];
    }
    vec[tmpack::kVU + e] = u;
    vec[tmpack::kVV + e] = v;
  }
  if (tid == 0) vec[tmpack::kVC] = static_cast<float>(c);
}

// ----------------------------------------------------------------------------------
// K1: persistent, warp-specialised LN_in + gated projections + mask -> a, b planes.
// Tile = 128 consecutive pairs (b, r, j0..j0+127); CTAs loop over tiles. 512 threads:
//   warps 0-7  LayerNorm producers, two threads per pair row (64 channels each, statistics
//              combined with one shuffle): one pass reads the staged, 128-B-swizzled z tile
//              into registers (conflict-free) and releases it, then the fp16 operand tile A
//              (xhat; the affine is folded into W1) is written and the pair's mask value
//              staged. (One thread per row with three passes over the tile kept the z
//              buffer busy through the whole LayerNorm.)
//              Thread 0 is also the TMA producer and MMA issuer: the 128 KB of packed
//              weights are loaded once; each tile's 128 x 128 fp32 z block arrives by TMA
//              (64 KB), refilled as soon as all producers have read it; after writing its
//              part of A it issues the tile's first-half MMAs, and the second half after
//              it has read the next tile's z (the issuing thread blocks on the tensor-core
//              queue, and the z refill waits for every producer). No warp is spent on
//              issuing alone, so sixteen warps keep 128 registers per thread.
//   warps 8-15 epilogue: thread = channel c (TMEM lane quarter = warp % 4), warps 8-11 take
//              pairs 0-63 of the tile and warps 12-15 pairs 64-127, in 16-pair chunks of the
//              projection / gate accumulators (the next chunk's TMEM loads in flight while
//              one is computed); each writes 32 contiguous bytes of its channel-plane row per
//              chunk. Two warps per scheduler: with one, the epilogue was latency-bound at
//              ~4,000 cycles per accumulator half (clock64 trace).
// MMA (transposed so that channels sit on TMEM lanes): D[c][j] = W_chunk[c][:] . A[j][:],
// M = 128 channels, N = 128 pairs, K = 128. Chunks (a_p, a_g) -> TMEM columns 0-255
// (half 0), (b_p, b_g) -> 256-511 (half 1); the epilogue of half 0 overlaps the MMAs of
// half 1, and the next tile's z load overlaps both.
// Gate: W1's gate rows and biases carry a factor 1/2 and the staged mask value is m/2, so
// with pm = (p + b_p) m / 2 the output is pm + pm tanh(g') = (p + b_p) sigmoid(g) m -- one
// MUFU op and three FP32 ops per element.
// Shared memory: W1 128 KB | A 32 KB | z 64 KB | mask 2 x 512 B | barriers.
// ----------------------------------------------------------------------------------
constexpr int kMaxPlaneDsts = 8;

namespace k1 {
constexpr int kThreads = 512;
constexpr uint32_t kW = 0, kA = 131072, kZ = 163840, kMask = 229376, kBar = 230400;
constexpr uint32_t kSmem = kBar + 128 + 1024;
static_assert(kSmem <= 232448, "K1 shared memory");
}  // namespace k1

// Destinations of the a / b planes. Channel c of pair row r goes to
// ptr[c / group] + (((b * dst_rows + row0 + r) * group + c % group) * ld) halves: with one
// group of 128 channels, dst_rows = rows and row0 = 0 this is the plain [B][rows][128][ld]
// layout; with P groups the planes land directly in the channel shards [B][dst_rows][128/P][ld]
// of P buffers (a peer GPU's memory mapped into this process, or local).
struct PlaneDsts {
  uint64_t ptr[kMaxPlaneDsts];
  int group, dst_rows, row0;
};

struct K1Bars {
  uint64_t wbar;
  uint64_t z_full, z_empty;
  uint64_t a_full, a_empty;
  uint64_t d_full[2], d_empty[2];
  uint64_t m_empty[2];
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K1Bars) <= 128, "K1 barrier block");

__global__ void __launch_bounds__(k1::kThreads, 1)
    trimul_project_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap z_map,
                          const float* __restrict__ mask, const float* __restrict__ vec,
                          const __grid_constant__ PlaneDsts a_dst, const __grid_constant__ PlaneDsts b_dst, int64_t ld,
                          int N, int rows, int n_jt, int n_tiles, uint32_t* status) {
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  K1Bars* bars = reinterpret_cast<K1Bars*>(smem + k1::kBar);
  CtaGuard* guard = &bars->guard;
  float* mask_s = reinterpret_cast<float*>(smem + k1::kMask);  // [2][128], m / 2
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
      mbar_init(&bars->m_empty[x], 256);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
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
    // ------- LayerNorm producers (two threads per pair row); thread 0 also issues -------
    // Each thread reads its 64 channels of the staged z tile into registers once and
    // releases the tile, so the next tile's z load overlaps the rest of the LayerNorm.
    const int p = warp * 16 + (lane >> 1), half = lane & 1;
    auto load_z = [&](int tile) {
      const int jt = tile % n_jt, rb = tile / n_jt;
      const int r = rb % rows, b = rb / rows;
      mbar_arrive_expect_tx(&bars->z_full, 65536);
#pragma unroll
      for (int q = 0; q < 4; ++q) tma_load_4d(smem + k1::kZ + q * 16384, &z_map, &bars->z_full, q * 32, jt * 128, r, b);
    };
    int loaded = 0;  // z tiles requested (thread 0)
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars->wbar, 131072);
#pragma unroll
      for (int kh = 0; kh < 2; ++kh)
#pragma unroll
        for (int rb = 0; rb < 4; ++rb)
          tma_load_2d(smem + k1::kW + kh * 65536 + rb * 16384, &w_map, &bars->wbar, kh * 64, rb * 128);
      load_z(blockIdx.x);  // the grid never exceeds the tile count
      loaded = 1;
    }
    const uint32_t idesc = make_idesc_f16(128, 128, 0, 0);
    const uint32_t w0 = smem_u32(smem + k1::kW), a0 = smem_u32(smem + k1::kA);
    // thread 0: the MMAs of accumulator half h of tile ti, once the epilogue has drained
    // half h of tile ti - 1; the second half also releases A
    auto issue_half = [&](int h, int ti) -> bool {
      if (ti >= 1 && !mbar_wait(&bars->d_empty[h], (ti - 1) & 1, guard, status, kStatusTimeoutMma)) return false;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int chunk = 2 * h + q;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int kh = ks >> 2, kin = ks & 3;
          umma_ss(tmem + h * 256 + q * 128, make_sdesc(w0 + kh * 65536 + chunk * 16384 + kin * 32, 16, 1024, Swz::k128),
                  make_sdesc(a0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128), idesc, ks > 0 ? 1u : 0u);
        }
      }
      umma_commit(&bars->d_full[h]);
      if (h == 1) umma_commit(&bars->a_empty);
      return true;
    };
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      const int jt = tile % n_jt, rb = tile / n_jt;
      const int r = rb % rows, b = rb / rows, j0 = jt * 128;
      // the pair's mask value, loaded before the waits so its DRAM latency is hidden
      float mval = 0.f;
      if (half == 0 && j0 + p < N)
        mval = mask ? __ldg(mask + (static_cast<size_t>(b) * rows + r) * N + j0 + p) : 1.f;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->z_full, it & 1, guard, status, kStatusTimeoutProducer));
      if (!ok) break;
      float v[64];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float4 t = lds_f4(smem + k1::kZ + (2 * half + q) * 16384 + swz128(p, ch));
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
        // the previous tile's second-half MMAs, issued only now that this tile's z has been
        // read: thread 0 blocks on the tensor-core queue while it issues, and with all of a
        // tile's MMAs issued before the next z read, the z refill (which waits for every
        // producer) started ~4,000 cycles later (clock64 trace)
        if (w && lane == 0 && it >= 1) w = issue_half(1, it - 1);
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
      bool w = true;
      if (it >= 1) w = mbar_wait(&bars->a_empty, (it - 1) & 1, guard, status, kStatusTimeoutProducer);
      if (it >= 2) w = w && mbar_wait(&bars->m_empty[s], ((it >> 1) - 1) & 1, guard, status, kStatusTimeoutProducer);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      if (half == 0) mask_s[s * 128 + p] = 0.5f * mval;
      // xhat only: gamma_in and beta_in are folded into W1 and b1
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int c = ch * 8;
        uint4 o;
        o.x = pack_f16x2((v[c + 0] - mean) * rstd, (v[c + 1] - mean) * rstd);
        o.y = pack_f16x2((v[c + 2] - mean) * rstd, (v[c + 3] - mean) * rstd);
        o.z = pack_f16x2((v[c + 4] - mean) * rstd, (v[c + 5] - mean) * rstd);
        o.w = pack_f16x2((v[c + 6] - mean) * rstd, (v[c + 7] - mean) * rstd);
        sts_u4(smem + k1::kA + half * 16384 + swz128(p, ch), o);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->a_full);
      if (warp == 0) {
        // thread 0: the tile's first-half MMAs (the second half follows the next z read)
        bool mw = true;
        if (lane == 0) {
          mw = mbar_wait(&bars->a_full, it & 1, guard, status, kStatusTimeoutMma);
          if (mw && it == 0) mw = mbar_wait(&bars->wbar, 0, guard, status, kStatusTimeoutMma);
          if (mw) mw = issue_half(0, it);
        }
        ok = __all_sync(0xffffffffu, mw);
        if (!ok) break;
      }
    }
    if (ok && warp == 0) {
      // the last tile's second half
      bool mw = true;
      if (lane == 0) mw = issue_half(1, it - 1);
      ok = __all_sync(0xffffffffu, mw);
    }
    if (!ok && tid == 0) {
      // abort: wait (bounded) for this thread's MMAs and TMA loads still in flight
      umma_commit(&bars->drain);
      mbar_wait_drain(&bars->drain, 0);
      if (loaded > 0) mbar_wait_drain(&bars->z_full, (loaded - 1) & 1);
      mbar_wait_drain(&bars->wbar, 0);
    }
  } else {
    // ------------------------- epilogue: thread = channel -------------------------
    const int q4 = warp & 3, jh = (warp - 8) >> 2;  // TMEM lane quarter, pair half of the tile
    const int c = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const int grp = c / a_dst.group, c_in_grp = c - grp * a_dst.group;  // this channel's destination group
    const float bias_p0 = vec[tmpack::kVB1 + c], bias_p1 = vec[tmpack::kVB1 + 256 + c];
    const float bias_g0 = vec[tmpack::kVB1 + 128 + c], bias_g1 = vec[tmpack::kVB1 + 384 + c];
    uint32_t sat = 0;  // an a / b value beyond the fp16 range was clamped
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      const int jt = tile % n_jt, rb = tile / n_jt;
      const int r = rb % rows, b = rb / rows, j0 = jt * 128 + jh * 64;
      const float* ms = mask_s + s * 128 + jh * 64;
      bool ok = true;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[h], it & 1, guard, status, kStatusTimeoutConsumer));
        if (!ok) break;
        tc_fence_after();
        // destination base re-read from the (constant-bank) parameters rather than kept live
        const uint64_t base = h ? b_dst.ptr[grp] : a_dst.ptr[grp];
        __half* dst = reinterpret_cast<__half*>(base) +
                      ((static_cast<size_t>(b) * a_dst.dst_rows + a_dst.row0 + r) * a_dst.group + c_in_grp) * ld;
        const bool wide = (ld & 15) == 0 && (base & 31) == 0;
        const float bp = h ? bias_p1 : bias_p0, bg = h ? bias_g1 : bias_g0;
        // 16-pair chunks of the projection / gate accumulators, software pipelined: the
        // TMEM loads of chunk k+1 are in flight while chunk k is computed and stored.
        const uint32_t tp = tmem + lane_off + h * 256 + jh * 64;
        uint32_t pv[2][16], gv[2][16];
        tmem_ld16(tp, pv[0]);
        tmem_ld16(tp + 128, gv[0]);
#pragma unroll
        for (int jc = 0; jc < 4; ++jc) {
          const int cur = jc & 1;
          tmem_wait_ld_regs(pv[cur], gv[cur]);
          if (jc + 1 < 4) {
            tmem_ld16(tp + (jc + 1) * 16, pv[cur ^ 1]);
            tmem_ld16(tp + 128 + (jc + 1) * 16, gv[cur ^ 1]);
          }
          uint32_t w[8];  // 16 pairs of this channel as fp16
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float4 m4 = *reinterpret_cast<const float4*>(ms + jc * 16 + u * 4);
            const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float pm = (__uint_as_float(pv[cur][u * 4 + e]) + bp) * mv[e];
              o[e] = fmaf(pm, tanh_approx(__uint_as_float(gv[cur][u * 4 + e]) + bg), pm);
            }
            w[2 * u] = pack_f16x2_chk(o[0], o[1], sat);
            w[2 * u + 1] = pack_f16x2_chk(o[2], o[3], sat);
          }
          // 32 contiguous bytes of the channel row: one 32-byte store when the plane pitch
          // keeps it 32-byte aligned (pitch a multiple of 16), two 16-byte stores otherwise
          const int jb = j0 + jc * 16;
          if (wide) {
            if (jb < ld) stg_v8(dst + jb, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]);
          } else {
#pragma unroll
            for (int v = 0; v < 2; ++v)
              if (jb + 8 * v < ld)
                *reinterpret_cast<uint4*>(dst + jb + 8 * v) = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&bars->d_empty[h]);
      }
      if (!ok) break;
      mbar_arrive(&bars->m_empty[s]);
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
// K2: per-channel contraction, persistent. One CTA per SM loops over output tiles of
// 128 rows (i) x 256 columns (j) of one (b, c) plane (j fastest, so consecutive tiles of a
// CTA wave share the A panel in L2). The K loop runs in blocks of 64 through a 4-stage TMA
// ring that continues across tiles; the accumulator is double buffered in TMEM
// (2 x 256 columns), so a tile's epilogue overlaps the next tile's MMAs. 192 threads:
//   warps 0-3  epilogue: thread = row (TMEM lane); TMEM -> fp16 (times out_scale) ->
//              two 16 KB staging buffers of 64 columns (128-B swizzle) -> TMA store;
//   warp 4     lane 0: TMA producer;
//   warp 5     lane 0: TMEM allocator and MMA issuer.
// (One tile per CTA, with the load latency up front and an epilogue that nothing
// overlapped, ran at 53% of the bf16 peak.)
// ----------------------------------------------------------------------------------
namespace k2 {
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr uint32_t kStageBytes = 49152;  // A 128x64 (16 KB) + B 256x64 (32 KB)
constexpr uint32_t kOut = kStages * kStageBytes;  // 2 staging buffers [128 rows][64 cols] fp16
constexpr uint32_t kBar = kOut + 2 * 16384;
constexpr uint32_t kSmem = kBar + 256 + 1024;
static_assert(kSmem <= 232448, "K2 shared memory");
}  // namespace k2

struct K2Bars {
  uint64_t full[k2::kStages], empty[k2::kStages];
  uint64_t d_full[2], d_empty[2];   // accumulator buffers: MMA commit / 128 epilogue threads
  uint64_t o_ready[2], o_free[2];   // staging halves: 128 epilogue threads / the storing thread
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K2Bars) <= 256, "K2 barrier block");

// Destinations of the peer form of K2 (the channel-sharded contraction of a row-sharded
// stack): the x tile of rows it*128.. goes to their owner p = it*128 / R, into p's x planes
// [B][R][C_dst][ld] at channel c_off + c. map[p] addresses them as (col, channel, row, b),
// box 64 columns x 1 channel x 128 rows: plain TMA stores into the peer's memory.
constexpr int kMaxK2Peers = 8;
struct K2Peers {
  CUtensorMap map[kMaxK2Peers];
  int R, c_off;
};

template <bool kOutgoing, bool kPeer>
__global__ void __launch_bounds__(k2::kThreads, 1)
    trimul_contract_kernel(const __grid_constant__ CUtensorMap a_map, const __grid_constant__ CUtensorMap b_map,
                           const __grid_constant__ CUtensorMap x_map, int C, int K, int n_jt, int n_it, int n_tiles,
                           float out_scale, uint32_t* status, const __grid_constant__ K2Peers peers) {
  using namespace k2;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  K2Bars* bars = reinterpret_cast<K2Bars*>(smem + kBar);
  CtaGuard* guard = &bars->guard;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB = (K + 63) / 64;
  auto decode = [&](int tile, int& jt, int& it, int& c, int& b) {
    jt = tile % n_jt;
    const int r = tile / n_jt;
    it = r % n_it;
    const int bc = r / n_it;
    c = bc % C;
    b = bc / C;
  };

  if (tid == 0) {
    guard->abort = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->d_full[x], 1);
      mbar_init(&bars->d_empty[x], 128);
      mbar_init(&bars->o_ready[x], 128);
      mbar_init(&bars->o_free[x], 1);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(&bars->tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;

  if (warp == 4) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int g = 0;  // global k-block counter (ring position)
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        int jt, it, c, b;
        decode(tile, jt, it, c, b);
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % kStages;
          if (g >= kStages &&
              !mbar_wait(&bars->empty[s], ((g / kStages) - 1) & 1, guard, status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + 16384;
          if (kOutgoing) {
            tma_load_4d(sa, &a_map, &bars->full[s], kb * 64, c, it * 128, b);
            tma_load_4d(sb, &b_map, &bars->full[s], kb * 64, c, jt * 256, b);
          } else {
#pragma unroll
            for (int h = 0; h < 2; ++h)
              tma_load_4d(sa + h * 8192, &a_map, &bars->full[s], it * 128 + h * 64, c, kb * 64, b);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              tma_load_4d(sb + q * 8192, &b_map, &bars->full[s], jt * 256 + q * 64, c, kb * 64, b);
          }
        }
      }
      if (!ok)  // after an abort, let the copies in flight land before shared memory is released
        for (int t = (g > kStages ? g - kStages : 0); t < g; ++t)
          mbar_wait_drain(&bars->full[t % kStages], (t / kStages) & 1);
    }
  } else if (warp == 5) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, 256, kOutgoing ? 0u : 1u, kOutgoing ? 0u : 1u);
      int g = 0, n = 0;  // k-block counter, tile counter of this CTA
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++n) {
        const int db = n & 1;
        if (n >= 2 && !mbar_wait(&bars->d_empty[db], ((n >> 1) - 1) & 1, guard, status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(&bars->full[s], (g / kStages) & 1, guard, status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kStageBytes);
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
            umma_ss(tmem + db * 256, ad, bd, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          umma_commit(&bars->empty[s]);
        }
        if (ok) umma_commit(&bars->d_full[db]);
      }
      umma_commit(&bars->drain);  // also drains whatever was issued before an abort
      mbar_wait_drain(&bars->drain, 0);
    }
  } else {
    // ------------------------- epilogue: thread = row -------------------------
    const int p = tid;  // warps 0-3
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const bool issuer = (tid == 0);
    bool ok = true;
    uint32_t sat = 0;     // an x value beyond the fp16 range was clamped
    int n = 0, half = 0;  // tile counter, staging-half counter
    for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++n) {
      int jt, it, c, b;
      decode(tile, jt, it, c, b);
      const int db = n & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[db], (n >> 1) & 1, guard, status, kStatusTimeoutConsumer));
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int hh = 0; hh < 4; ++hh, ++half) {
        // staging buffer: columns hh*64 .. +63 as one box of [128 rows][128 B]
        const int ob = half & 1;
        if (half >= 2) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_free[ob], ((half >> 1) - 1) & 1, guard, status,
                                                 kStatusTimeoutConsumer));
          if (!ok) break;
        }
        uint8_t* stage = smem + kOut + ob * 16384;
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + db * 256 + hh * 64 + cc * 32, v);
          tmem_wait_ld();
          uint8_t* box = stage;
          const int chb = cc * 4;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 o;
            o.x = pack_f16x2_chk(__uint_as_float(v[u * 8 + 0]) * out_scale, __uint_as_float(v[u * 8 + 1]) * out_scale,
                                 sat);
            o.y = pack_f16x2_chk(__uint_as_float(v[u * 8 + 2]) * out_scale, __uint_as_float(v[u * 8 + 3]) * out_scale,
                                 sat);
            o.z = pack_f16x2_chk(__uint_as_float(v[u * 8 + 4]) * out_scale, __uint_as_float(v[u * 8 + 5]) * out_scale,
                                 sat);
            o.w = pack_f16x2_chk(__uint_as_float(v[u * 8 + 6]) * out_scale, __uint_as_float(v[u * 8 + 7]) * out_scale,
                                 sat);
            sts_u4(box + swz128(p, chb + u), o);
          }
        }
        if (hh == 3) {
          tc_fence_before();
          mbar_arrive(&bars->d_empty[db]);  // the accumulator buffer is read: next MMAs may start
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->o_ready[ob]);
        if (warp == 0) {
          // one thread stores the half once all 128 have written it (bounded waits, so that an
          // abort elsewhere cannot leave threads parked at a barrier)
          bool iok = true;
          if (issuer) {
            iok = mbar_wait(&bars->o_ready[ob], (half >> 1) & 1, guard, status, kStatusTimeoutConsumer);
            if (iok) {
              if constexpr (kPeer) {
                const int p = (it * 128) / peers.R;
                tma_store_4d(&peers.map[p], stage, jt * 256 + hh * 64, peers.c_off + c, it * 128 - p * peers.R, b);
              } else {
                tma_store_4d(&x_map, stage, jt * 256 + hh * 64, c, it * 128, b);
              }
              tma_store_commit();
              tma_store_wait_read();
              mbar_arrive(&bars->o_free[ob]);
            }
          }
          ok = __shfl_sync(0xffffffffu, iok ? 1 : 0, 0) != 0;
        }
        if (!ok) break;
      }
    }
    if (issuer) tma_store_wait_all();
    flag_saturation(sat, status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------------
// K2e: persistent LN_out + linear_z + output gate (+ residual). Tile = 128 consecutive
// pairs; CTAs loop over tiles. 608 threads:
//   warps 0-7   LayerNorm producers for the gate: LN_in(z) of the tile's pairs, two threads
//               per pair (64 channels each, combined with one shuffle), read from the
//               TMA-staged z tile into registers and, once all 256 have read it, written as
//               the fp16 operand A over the first half of the same buffer;
//   warps 8-15  epilogue: thread = pair p (TMEM lane), two warps per lane quarter; each
//               takes the pair's LN_out statistics from the x tile in shared memory, then
//               warps 8-11 finish the 32-channel slabs 0 and 1 and warps 12-15 slabs 2 and 3:
//               the residual slab of z arrives by TMA, is updated in place with
//               gate * linear_z(LN_out(x)) and leaves by TMA store (one buffer per slab, so
//               the next tile's residual loads run ahead), so every global access is a bulk
//               tensor copy. (With one epilogue warp per scheduler, warps 8-11 only, the
//               epilogue was the critical path at ~9,800 cycles per tile, clock64 trace.)
//   warp 16     lane 0: MMA issuer;
//   warp 17     lane 0: TMA for the weights (once), the z tile and the x tile;
//   warp 18     lane 0: slab manager -- TMA loads of the residual slabs and TMA stores of
//               the finished ones (a slab buffer is reloaded once its store has read it).
// TMEM (double buffered per tile, 256 columns each): G = A W_g^T at +0, U = x^T (W_z gamma)^T
// at +128. LN_out folds into the epilogue: out = g * (rstd (U - mu u) + v), with the gate
// g = (1 + tanh(G + b_g')) / 2 (W_g's rows and b_g' carry the 1/2 of sigmoid(x) = (1 + tanh(x/2)) / 2).
// Shared memory: W2 64 KB | z tile / A 64 KB | x 32 KB | slabs 4 x 16 KB | b_g,u,v | barriers.
// The z tile is reloaded once the gate GEMM has read A from the same buffer.
// (A warp-per-pair LayerNorm read from global memory and per-thread residual loads, each
// warp load touching 32 separate pairs, held this kernel at ~17k cycles per tile.)
// ----------------------------------------------------------------------------------
namespace k2e {
constexpr int kThreads = 608;
constexpr int kSlabs = 4;
constexpr uint32_t kW = 0, kZ = 65536, kA = kZ, kX = 131072, kO = 163840, kVec = 229376, kBar = 229376 + 1536;
constexpr uint32_t kSmem = kBar + 256 + 1024;
static_assert(kO + kSlabs * 16384 <= kVec, "K2e slabs");
static_assert(kSlabs == 4, "one slab buffer per 32-channel slab of a tile");
static_assert(kSmem <= 232448, "K2e shared memory");
}  // namespace k2e

struct K2eBars {
  uint64_t wbar;
  uint64_t z_full, z_read;   // z tile: TMA / all 256 LayerNorm threads have read it
  uint64_t a_full, a_empty;  // 256 LayerNorm threads / MMA commit (the z tile may be reloaded)
  uint64_t x_full, x_empty;  // TMA / MMA commit + 128 epilogue threads (statistics)
  uint64_t d_full[2], d_empty[2];
  uint64_t o_full[k2e::kSlabs];      // residual slab landed (TMA) / buffer handed to the epilogue
  uint64_t slab_ready[k2e::kSlabs];  // 128 epilogue threads wrote the slab
  uint64_t drain;
  uint32_t tslot;
  CtaGuard guard;
};
static_assert(sizeof(K2eBars) <= 256, "K2e barrier block");

// kDrop: the update is multiplied by the channel dropout `drop` before the residual add
// (out = z + keep * scale * update); the plain instantiation ignores `drop`.
template <bool kDrop>
__global__ void __launch_bounds__(k2e::kThreads, 1)
    trimul_finish_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map,
                         const __grid_constant__ CUtensorMap z_map, const __grid_constant__ CUtensorMap out_map,
                         const float* __restrict__ vec, int add_residual, float x_scale, int N, int rows, int n_jt,
                         int n_tiles, uint32_t* status, const DropArgs drop) {
  using namespace k2e;
  const float c_real = __ldg(vec + tmpack::kVC);  // real hidden channels (<= 128)
  const float n_pad = 128.f - c_real, inv_c = 1.f / c_real;
  extern __shared__ uint8_t dsmem[];
  uint8_t* smem = align1024(dsmem);
  K2eBars* bars = reinterpret_cast<K2eBars*>(smem + kBar);
  CtaGuard* guard = &bars->guard;
  float* svec = reinterpret_cast<float*>(smem + kVec);  // b_g | u | v
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    guard->abort = 0;
    mbar_init(&bars->wbar, 1);
    mbar_init(&bars->z_full, 1);
    mbar_init(&bars->z_read, 256);
    mbar_init(&bars->a_full, 256);
    mbar_init(&bars->a_empty, 1);
    mbar_init(&bars->x_full, 1);
    mbar_init(&bars->x_empty, 1 + 256);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->d_full[x], 1);
      mbar_init(&bars->d_empty[x], 256);
    }
    for (int x = 0; x < kSlabs; ++x) {
      mbar_init(&bars->o_full[x], 1);
      mbar_init(&bars->slab_ready[x], 128);
    }
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (tid < 128) {
    svec[tid] = vec[tmpack::kVBg + tid];
    svec[128 + tid] = vec[tmpack::kVU + tid];
    svec[256 + tid] = vec[tmpack::kVV + tid];
  }
  if (warp == 16) {
    tmem_alloc(&bars->tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tslot;

  if (warp < 8) {
    // ---------------- LayerNorm producers: two threads per pair row ----------------
    const int row = warp * 16 + (lane >> 1), half = lane & 1;
    int it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->z_full, it & 1, guard, status, kStatusTimeoutProducer))) break;
      // channels 64*half .. 64*half+63 are boxes 2*half, 2*half+1 of the staged tile
      float v[64];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const float4 t = lds_f4(smem + kZ + (2 * half + q) * 16384 + swz128(row, ch));
          v[q * 32 + ch * 4 + 0] = t.x;
          v[q * 32 + ch * 4 + 1] = t.y;
          v[q * 32 + ch * 4 + 2] = t.z;
          v[q * 32 + ch * 4 + 3] = t.w;
        }
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) s4[c & 3] += v[c];
      float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      // the tile is released (A is written over it, the next z half is loaded into it) once
      // every loaded value has been consumed, see mbar_arrive_after
      mbar_arrive_after(&bars->z_read, sum);
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
      // A overwrites the z tile: wait until every LayerNorm thread has read its rows
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->z_read, it & 1, guard, status, kStatusTimeoutProducer))) break;
      // xhat only: gamma_in and beta_in are folded into the gate weights and b_g
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int c = ch * 8;
        uint4 o;
        o.x = pack_f16x2((v[c + 0] - mean) * rstd, (v[c + 1] - mean) * rstd);
        o.y = pack_f16x2((v[c + 2] - mean) * rstd, (v[c + 3] - mean) * rstd);
        o.z = pack_f16x2((v[c + 4] - mean) * rstd, (v[c + 5] - mean) * rstd);
        o.w = pack_f16x2((v[c + 6] - mean) * rstd, (v[c + 7] - mean) * rstd);
        sts_u4(smem + kA + half * 16384 + swz128(row, ch), o);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->a_full);
    }
  } else if (warp == 16) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(&bars->wbar, 0, guard, status, kStatusTimeoutMma);
      const uint32_t id_g = make_idesc_f16(128, 128, 0, 0);
      const uint32_t id_u = make_idesc_f16(128, 128, 1, 0);
      const uint32_t w0 = smem_u32(smem + kW);
      const uint32_t a0 = smem_u32(smem + kA), x0 = smem_u32(smem + kX);
      int it = 0;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
        const int s = it & 1;
        ok = mbar_wait(&bars->a_full, it & 1, guard, status, kStatusTimeoutMma);
        ok = ok && mbar_wait(&bars->x_full, it & 1, guard, status, kStatusTimeoutMma);
        if (ok && it >= 2) ok = mbar_wait(&bars->d_empty[s], ((it >> 1) - 1) & 1, guard, status, kStatusTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + s * 256;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int kh = ks >> 2, kin = ks & 3;
          umma_ss(d, make_sdesc(a0 + kh * 16384 + kin * 32, 16, 1024, Swz::k128),
                  make_sdesc(w0 + kh * 32768 + kin * 32, 16, 1024, Swz::k128), id_g, ks > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int kh = ks >> 2, kin = ks & 3;
          umma_ss(d + 128, make_sdesc(x0 + ks * 2048, 16384, 1024, Swz::k128),
                  make_sdesc(w0 + kh * 32768 + 16384 + kin * 32, 16, 1024, Swz::k128), id_u, ks > 0 ? 1u : 0u);
        }
        umma_commit(&bars->d_full[s]);
        umma_commit(&bars->a_empty);
        umma_commit(&bars->x_empty);
      }
      if (!ok) {
        umma_commit(&bars->drain);
        mbar_wait_drain(&bars->drain, 0);
      }
    }
  } else if (warp == 17) {
    // ------------------- TMA producer: weights, z tiles, x tiles -------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars->wbar, 65536);
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) tma_load_2d(smem + kW + kh * 32768, &w_map, &bars->wbar, kh * 64, 0);
      bool ok = true;
      int it = 0, zl = 0, xl = 0;  // z / x tiles loaded
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const int jt = tile % n_jt, rb = tile / n_jt;
        const int r = rb % rows, b = rb / rows, j0 = jt * 128;
        // Channels 64-127 (boxes 2, 3) as soon as every LayerNorm thread has read the previous
        // tile (A never covers them); channels 0-63 once the gate GEMM has read A, which
        // overwrites them. Only the second half of the load sits between that GEMM and the
        // next LayerNorm.
        if (it >= 1 && !mbar_wait(&bars->z_read, (it - 1) & 1, guard, status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&bars->z_full, 32768);
#pragma unroll
        for (int q = 2; q < 4; ++q) tma_load_4d(smem + kZ + q * 16384, &z_map, &bars->z_full, q * 32, j0, r, b);
        ++zl;
        if (it >= 1 && !mbar_wait(&bars->a_empty, (it - 1) & 1, guard, status, kStatusTimeoutProducer)) {
          mbar_arrive(&bars->z_full);  // complete the phase on the half in flight, so the drain below can wait for it
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->z_full, 32768);
#pragma unroll
        for (int q = 0; q < 2; ++q) tma_load_4d(smem + kZ + q * 16384, &z_map, &bars->z_full, q * 32, j0, r, b);
        if (it >= 1 && !mbar_wait(&bars->x_empty, (it - 1) & 1, guard, status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->x_full, 32768);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          tma_load_4d(smem + kX + hh * 16384, &x_map, &bars->x_full, j0 + hh * 64, 0, r, b);
        ++xl;
      }
      // after an abort, let the last copies land before the CTA's shared memory is released
      if (!ok) {
        if (zl > 0) mbar_wait_drain(&bars->z_full, (zl - 1) & 1);
        if (xl > 0) mbar_wait_drain(&bars->x_full, (xl - 1) & 1);
      }
      mbar_wait_drain(&bars->wbar, 0);
    }
  } else if (warp == 18) {
    // ---------------- slab manager: residual loads and output stores ----------------
    // Slab sn (four per tile, 32 channels each) lives in buffer sn % 4. Its output store is
    // issued once the 128 epilogue threads have written it; once that store has read the
    // buffer, the residual of slab sn + 4 (the next tile's slab of the same channels) is
    // loaded into it. Issuing here keeps the store and its wait off the epilogue warps.
    if (lane == 0) {
      bool ok = true;
      const int n_mine = (n_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
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
  } else {
    // ------------------------- epilogue: thread = pair -------------------------
    // Two warps per TMEM lane quarter: warps 8-11 finish slabs 0, 1 (channels 0-63) and
    // warps 12-15 slabs 2, 3 of every tile; both take the pair's LN_out statistics.
    const int q4 = warp & 3, hh = (warp - 8) >> 2;
    const int p = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++it) {
      const int s = it & 1;
      uint4 keep = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (kDrop) {  // issued before the waits so that its latency hides under them
        const int jt = tile % n_jt, rb = tile / n_jt;
        keep = drop_keep(drop, rb / rows, rb % rows, jt * 128 + p, N);
      }
      bool w = mbar_wait(&bars->x_full, it & 1, guard, status, kStatusTimeoutConsumer);
      w = w && mbar_wait(&bars->d_full[s], (it >> 1) & 1, guard, status, kStatusTimeoutConsumer);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      // LN_out statistics over the c_real channels of pair p (x is stored times x_scale). The
      // channels past c_real of a narrower update are exact zeros: the loop runs over all 128
      // (a constant trip count keeps the chains in registers) and the n_pad zero channels'
      // terms, -x0 and x0^2 each, are taken out again (nothing to take out at 128 channels).
      const uint8_t* xb = smem + kX + (p >> 6) * 16384;
      const int pj = p & 63;
      const float x0 = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(xb + swz128(0, pj >> 3) + (pj & 7) * 2)));
      float a1[4] = {0.f, 0.f, 0.f, 0.f}, a2[4] = {0.f, 0.f, 0.f, 0.f};  // four chains each
#pragma unroll 16
      for (int c = 0; c < 128; ++c) {
        const float xv = __half2float(
                             __ushort_as_half(*reinterpret_cast<const uint16_t*>(xb + swz128(c, pj >> 3) + (pj & 7) * 2))) -
                         x0;
        a1[c & 3] += xv;
        a2[c & 3] = fmaf(xv, xv, a2[c & 3]);
      }
      const float s1 = ((a1[0] + a1[1]) + (a1[2] + a1[3])) + n_pad * x0;
      const float s2 = ((a2[0] + a2[1]) + (a2[2] + a2[3])) - n_pad * x0 * x0;
      mbar_arrive_after(&bars->x_empty, s1 + s2);  // the x tile may be reloaded: its values are consumed
      const float d1 = s1 * inv_c;
      const float mu_x = x0 + d1;
      const float var = fmaxf(s2 * inv_c - d1 * d1, 0.f);
      const float rstd_x = rsqrtf(var + 1e-5f * x_scale * x_scale);
      tc_fence_after();
#pragma unroll 1
      for (int cc = 2 * hh; cc < 2 * hh + 2; ++cc) {
        const int sl = cc;  // slab it * 4 + cc of this CTA lives in buffer cc
        uint32_t g[32], u[32];
        tmem_ld32(tmem + lane_off + s * 256 + cc * 32, g);
        tmem_ld32(tmem + lane_off + s * 256 + 128 + cc * 32, u);
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->o_full[sl], it & 1, guard, status,
                                               kStatusTimeoutConsumer));
        tmem_wait_ld();
        if (!ok) break;
        uint8_t* ob = smem + kO + sl * 16384;
        const uint32_t kw = kDrop ? drop_word(keep, cc) : 0u;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float o[4];
          const int n0 = cc * 32 + q * 4;
          const float4 zv = add_residual ? lds_f4(ob + swz128(p, q)) : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 bg4 = *reinterpret_cast<const float4*>(svec + n0);
          const float4 u4 = *reinterpret_cast<const float4*>(svec + 128 + n0);
          const float4 v4 = *reinterpret_cast<const float4*>(svec + 256 + n0);
          const float rq[4] = {zv.x, zv.y, zv.z, zv.w};
          const float bgv[4] = {bg4.x, bg4.y, bg4.z, bg4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w},
                      vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int t = q * 4 + e;
            const float gate = fmaf(0.5f, tanh_approx(__uint_as_float(g[t]) + bgv[e]), 0.5f);
            const float y = fmaf(rstd_x, fmaf(-mu_x, uv[e], __uint_as_float(u[t])), vv[e]);
            if constexpr (kDrop) {
              const float ds = ((kw >> t) & 1u) ? drop.scale : 0.f;
              o[e] = fmaf(y * gate, ds, rq[e]);
            } else {
              o[e] = fmaf(y, gate, rq[e]);
            }
          }
          *reinterpret_cast<float4*>(ob + swz128(p, q)) = make_float4(o[0], o[1], o[2], o[3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->slab_ready[sl]);  // warp 18 stores the slab
      }
      if (!ok) break;
      tc_fence_before();
      mbar_arrive(&bars->d_empty[s]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 16) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------------
// ----------------------------------------------------------------------------------
// Built-in scratch for gtk_trimul_forward_noalloc: room for the a, b and x planes of
// one call (3 * B * N * round_up(N, 8) * 128 fp16 values). It is allocated once per GPU
// when the library's kernels are first loaded there and lives until the process exits.
// ----------------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(24) << 20;
static __device__ __align__(256) uint8_t g_trimul_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array on the current device, looked up once per device.
// Host code must not use the array's name as a device pointer: on the host it names a
// shadow variable, not device memory.
static int noalloc_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(GTK_ERR_CUDA, "trimul_forward_noalloc: no usable current device");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_trimul_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(GTK_ERR_CUDA, std::string("trimul_forward_noalloc: cudaGetSymbolAddress failed: ") +
                                    cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return GTK_OK;
}

}  // namespace gtk

using namespace gtk;

extern "C" {

// The tuned kernels: c_z = 128 and c_hidden <= 128 (a narrower hidden width zero-padded to 128
// channels when packed).
static bool trimul_tuned(int c_z, int c_hidden) { return c_z == 128 && c_hidden >= 1 && c_hidden <= 128; }

size_t gtk_trimul_packed_bytes(int c_z, int c_hidden) {
  if (!trimul_tuned(c_z, c_hidden)) return gen::trimul_packed_bytes(c_z, c_hidden);
  return tmpack::kBytes;
}

int gtk_trimul_pack(const gtk_trimul_params* params, int c_z, int c_hidden, void* packed, size_t packed_bytes,
                    void* stream) {
  if (!trimul_tuned(c_z, c_hidden)) return gen::trimul_pack(params, c_z, c_hidden, packed, packed_bytes, stream);
  if (!params) return fail(GTK_ERR_INVALID_ARG, "params is NULL");
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (packed_bytes < tmpack::kBytes) return fail(GTK_ERR_WORKSPACE, "packed buffer too small");
  const float* const* pp = reinterpret_cast<const float* const*>(params);
  for (int i = 0; i < 16; ++i)
    if (!pp[i]) return fail(GTK_ERR_INVALID_ARG, "a trimul parameter pointer is NULL");
  if (int e = check_device()) return e;
  trimul_pack_kernel<<<64, 256, 0, static_cast<cudaStream_t>(stream)>>>(*params, static_cast<uint8_t*>(packed),
                                                                         c_hidden);
  return check_launch("trimul_pack_kernel");
}

int64_t gtk_plane_pitch(int64_t N) { return static_cast<int64_t>(round_up(static_cast<uint64_t>(N), 8)); }

size_t gtk_trimul_workspace_bytes(int64_t B, int64_t N, int c_z, int c_hidden) {
  if (!trimul_tuned(c_z, c_hidden)) return gen::trimul_workspace_bytes(B, N, c_z, c_hidden);
  if (B < 1 || N < 1) return 0;
  const size_t plane = round_up(static_cast<size_t>(B) * N * 128 * gtk_plane_pitch(N) * 2, 256);
  return 3 * plane;
}

static int trimul_project_launch(const float* z, const float* mask, const void* packed, const PlaneDsts& ad,
                                 const PlaneDsts& bd, int64_t ld, int64_t B, int64_t rows, int64_t N,
                                 uint32_t* status, void* stream) {
  if (!dims_ok(B, 65535) || !dims_ok(rows, 65535) || !dims_ok(N, 1 << 20))
    return fail(GTK_ERR_INVALID_ARG, "trimul_project: bad B/rows/N");
  if (ld < N || ld % 8) return fail(GTK_ERR_INVALID_ARG, "trimul_project: plane pitch must be >= N and a multiple of 8");
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (mask && (reinterpret_cast<uintptr_t>(mask) & 3)) return fail(GTK_ERR_ALIGNMENT, "mask is misaligned");
  if (int e = check_device()) return e;
  const int64_t n_jt = (N + 127) / 128;
  const int64_t n_tiles = B * rows * n_jt;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "trimul_project: too many tiles");
  CUtensorMap wm, zm;
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  if (int e = make_weight_map(&wm, pk + tmpack::kW1, 512, 128)) return e;
  if (int e = make_pair_map(&zm, z, B, rows, N, false)) return e;
  if (int e = ensure_smem(reinterpret_cast<const void*>(trimul_project_kernel), k1::kSmem)) return e;
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  trimul_project_kernel<<<grid, k1::kThreads, k1::kSmem, static_cast<cudaStream_t>(stream)>>>(
      wm, zm, mask, reinterpret_cast<const float*>(pk + tmpack::kVec), ad, bd, ld, static_cast<int>(N),
      static_cast<int>(rows), static_cast<int>(n_jt), static_cast<int>(n_tiles), status);
  return check_launch("trimul_project_kernel");
}

int gtk_trimul_project(const float* z, const float* mask, const void* packed, void* a_planes, void* b_planes,
                       int64_t ld, int64_t B, int64_t rows, int64_t N, uint32_t* status, void* stream) {
  if (int e = check_ptr(a_planes, "a_planes")) return e;
  if (int e = check_ptr(b_planes, "b_planes")) return e;
  PlaneDsts ad{}, bd{};
  ad.ptr[0] = reinterpret_cast<uint64_t>(a_planes);
  bd.ptr[0] = reinterpret_cast<uint64_t>(b_planes);
  ad.group = bd.group = 128;
  ad.dst_rows = bd.dst_rows = static_cast<int>(rows);
  ad.row0 = bd.row0 = 0;
  return trimul_project_launch(z, mask, packed, ad, bd, ld, B, rows, N, status, stream);
}

int gtk_trimul_project_sharded(const float* z, const float* mask, const void* packed, void* const* a_dsts,
                               void* const* b_dsts, int P, int64_t dst_rows, int64_t row0, int64_t ld, int64_t B,
                               int64_t rows, int64_t N, uint32_t* status, void* stream) {
  if (P < 1 || P > kMaxPlaneDsts || 128 % P)
    return fail(GTK_ERR_INVALID_ARG, "trimul_project_sharded: P must divide 128 and be at most 8");
  if (!a_dsts || !b_dsts) return fail(GTK_ERR_INVALID_ARG, "trimul_project_sharded: NULL destination table");
  if (row0 < 0 || row0 + rows > dst_rows || dst_rows > 65535)
    return fail(GTK_ERR_INVALID_ARG, "trimul_project_sharded: rows row0..row0+rows must lie in dst_rows");
  PlaneDsts ad{}, bd{};
  for (int q = 0; q < P; ++q) {
    if (int e = check_ptr(a_dsts[q], "a_dsts[q]")) return e;
    if (int e = check_ptr(b_dsts[q], "b_dsts[q]")) return e;
    ad.ptr[q] = reinterpret_cast<uint64_t>(a_dsts[q]);
    bd.ptr[q] = reinterpret_cast<uint64_t>(b_dsts[q]);
  }
  ad.group = bd.group = 128 / P;
  ad.dst_rows = bd.dst_rows = static_cast<int>(dst_rows);
  ad.row0 = bd.row0 = static_cast<int>(row0);
  return trimul_project_launch(z, mask, packed, ad, bd, ld, B, rows, N, status, stream);
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
  const void* kern = outgoing ? reinterpret_cast<const void*>(trimul_contract_kernel<true, false>)
                              : reinterpret_cast<const void*>(trimul_contract_kernel<false, false>);
  if (int e = ensure_smem(kern, k2::kSmem)) return e;
  const int64_t n_jt = (Nj + 255) / 256, n_it = (M + 127) / 128;
  const int64_t n_tiles = n_jt * n_it * B * C;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "trimul_contract: too many tiles");
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const K2Peers none{};
  if (outgoing)
    trimul_contract_kernel<true, false><<<grid, k2::kThreads, k2::kSmem, st>>>(
        am, bm, xm, static_cast<int>(C), static_cast<int>(K), static_cast<int>(n_jt), static_cast<int>(n_it),
        static_cast<int>(n_tiles), out_scale, status, none);
  else
    trimul_contract_kernel<false, false><<<grid, k2::kThreads, k2::kSmem, st>>>(
        am, bm, xm, static_cast<int>(C), static_cast<int>(K), static_cast<int>(n_jt), static_cast<int>(n_it),
        static_cast<int>(n_tiles), out_scale, status, none);
  return check_launch("trimul_contract_kernel");
}

int gtk_trimul_contract_to_peers(int outgoing, const void* a_planes, const void* b_planes, const uint64_t* dst_bases,
                                 int P, int64_t B, int64_t C, int64_t M, int64_t Nj, int64_t K, int64_t lda,
                                 int64_t ldb, int64_t C_dst, int64_t c_off, int64_t ld_dst, float out_scale,
                                 uint32_t* status, void* stream) {
  if (P < 1 || P > kMaxK2Peers || !dst_bases) return fail(GTK_ERR_INVALID_ARG, "trimul_contract_to_peers: bad P");
  if (!dims_ok(B) || !dims_ok(C) || !dims_ok(M) || !dims_ok(Nj) || !dims_ok(K) || B * C > 65535 * 1024 ||
      c_off < 0 || c_off + C > C_dst || M % P)
    return fail(GTK_ERR_INVALID_ARG, "trimul_contract_to_peers: bad sizes");
  const int64_t R = M / P;
  if (R % 128) return fail(GTK_ERR_UNSUPPORTED, "trimul_contract_to_peers: rows per rank must be a multiple of 128");
  if (lda % 8 || ldb % 8 || ld_dst % 8) return fail(GTK_ERR_ALIGNMENT, "trimul_contract_to_peers: pitches must be multiples of 8");
  if (outgoing ? (lda < K || ldb < K) : (lda < M || ldb < Nj)) return fail(GTK_ERR_INVALID_ARG, "pitch too small");
  if (ld_dst < Nj) return fail(GTK_ERR_INVALID_ARG, "trimul_contract_to_peers: ld_dst < Nj");
  if (int e = check_ptr(a_planes, "a_planes")) return e;
  if (int e = check_ptr(b_planes, "b_planes")) return e;
  for (int p = 0; p < P; ++p)
    if (int e = check_ptr(reinterpret_cast<const void*>(dst_bases[p]), "peer x planes")) return e;
  if (int e = check_device()) return e;
  CUtensorMap am, bm;
  if (outgoing) {
    if (int e = make_plane_map(&am, a_planes, B, M, C, K, lda, 64, 1, 128, 128)) return e;
    if (int e = make_plane_map(&bm, b_planes, B, Nj, C, K, ldb, 64, 1, 256, 128)) return e;
  } else {
    if (int e = make_plane_map(&am, a_planes, B, K, C, M, lda, 64, 1, 64, 128)) return e;
    if (int e = make_plane_map(&bm, b_planes, B, K, C, Nj, ldb, 64, 1, 64, 128)) return e;
  }
  K2Peers peers{};
  peers.R = static_cast<int>(R);
  peers.c_off = static_cast<int>(c_off);
  for (int p = 0; p < P; ++p)
    if (int e = make_plane_map(&peers.map[p], reinterpret_cast<const void*>(dst_bases[p]), B, R, C_dst, Nj, ld_dst, 64,
                               1, 128, 128))
      return e;
  const void* kern = outgoing ? reinterpret_cast<const void*>(trimul_contract_kernel<true, true>)
                              : reinterpret_cast<const void*>(trimul_contract_kernel<false, true>);
  if (int e = ensure_smem(kern, k2::kSmem)) return e;
  const int64_t n_jt = (Nj + 255) / 256, n_it = M / 128;
  const int64_t n_tiles = n_jt * n_it * B * C;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "trimul_contract_to_peers: too many tiles");
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (outgoing)
    trimul_contract_kernel<true, true><<<grid, k2::kThreads, k2::kSmem, st>>>(
        am, bm, am, static_cast<int>(C), static_cast<int>(K), static_cast<int>(n_jt), static_cast<int>(n_it),
        static_cast<int>(n_tiles), out_scale, status, peers);
  else
    trimul_contract_kernel<false, true><<<grid, k2::kThreads, k2::kSmem, st>>>(
        am, bm, am, static_cast<int>(C), static_cast<int>(K), static_cast<int>(n_jt), static_cast<int>(n_it),
        static_cast<int>(n_tiles), out_scale, status, peers);
  return check_launch("trimul_contract_kernel (to peers)");
}

}  // extern "C"

namespace gtk {

// K2e launch; `drop` with a NULL keep array selects the plain instantiation.
static int trimul_finish_launch(const float* z, const void* x_planes, int64_t ldx, float x_scale, const void* packed,
                                float* out, int add_residual, int64_t B, int64_t rows, int64_t N, uint32_t* status,
                                void* stream, const DropArgs& drop) {
  if (!dims_ok(B, 65535) || !dims_ok(rows, 65535) || !dims_ok(N, 1 << 20))
    return fail(GTK_ERR_INVALID_ARG, "trimul_finish: bad B/rows/N");
  if (ldx < N || ldx % 8) return fail(GTK_ERR_INVALID_ARG, "trimul_finish: bad plane pitch");
  if (!(x_scale > 0.f)) return fail(GTK_ERR_INVALID_ARG, "trimul_finish: x_scale must be positive");
  if (int e = check_ptr(z, "z")) return e;
  if (int e = check_ptr(out, "out")) return e;
  if (int e = check_ptr(x_planes, "x_planes")) return e;
  if (int e = check_ptr(packed, "packed", 256)) return e;
  if (int e = check_device()) return e;
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
  const int64_t n_jt = (N + 127) / 128;
  const int64_t n_tiles = B * rows * n_jt;
  if (n_tiles > 2147483647) return fail(GTK_ERR_INVALID_ARG, "trimul_finish: too many tiles");
  CUtensorMap wm, xm, zm, om;
  if (int e = make_weight_map(&wm, pk + tmpack::kW2, 256, 256)) return e;
  if (int e = make_plane_map(&xm, x_planes, B, rows, 128, N, ldx, 64, 128, 1, 128)) return e;
  if (int e = make_pair_map(&zm, z, B, rows, N, false)) return e;
  if (int e = make_pair_map(&om, out, B, rows, N, false)) return e;
  const bool dropping = drop.keep != nullptr;
  const void* kern = dropping ? reinterpret_cast<const void*>(trimul_finish_kernel<true>)
                              : reinterpret_cast<const void*>(trimul_finish_kernel<false>);
  if (int e = ensure_smem(kern, k2e::kSmem)) return e;
  const int grid = static_cast<int>(n_tiles < num_sms() ? n_tiles : num_sms());
  const float* vec = reinterpret_cast<const float*>(pk + tmpack::kVec);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dropping)
    trimul_finish_kernel<true><<<grid, k2e::kThreads, k2e::kSmem, st>>>(
        wm, xm, zm, om, vec, add_residual, x_scale, static_cast<int>(N), static_cast<int>(rows),
        static_cast<int>(n_jt), static_cast<int>(n_tiles), status, drop);
  else
    trimul_finish_kernel<false><<<grid, k2e::kThreads, k2e::kSmem, st>>>(
        wm, xm, zm, om, vec, add_residual, x_scale, static_cast<int>(N), static_cast<int>(rows),
        static_cast<int>(n_jt), static_cast<int>(n_tiles), status, drop);
  return check_launch("trimul_finish_kernel");
}

static int trimul_forward_impl(int outgoing, const float* z, const float* mask, const void* packed, float* out,
                               int add_residual, const DropArgs& drop, void* workspace, size_t workspace_bytes,
                               int64_t B, int64_t N, int c_z, int c_hidden, uint32_t* status, void* stream) {
  if (!trimul_tuned(c_z, c_hidden))  // every other shape: the general path
    return gen::trimul_forward(outgoing, z, mask, packed, out, add_residual, drop, workspace, workspace_bytes, B, N,
                               c_z, c_hidden, status, stream);
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
  return trimul_finish_launch(z, xp, ld, xs, packed, out, add_residual, B, N, N, status, stream, drop);
}

}  // namespace gtk

extern "C" {

int gtk_trimul_finish(const float* z, const void* x_planes, int64_t ldx, float x_scale, const void* packed,
                      float* out, int add_residual, int64_t B, int64_t rows, int64_t N, uint32_t* status,
                      void* stream) {
  return trimul_finish_launch(z, x_planes, ldx, x_scale, packed, out, add_residual, B, rows, N, status, stream,
                              DropArgs{});
}

int gtk_trimul_forward(int outgoing, const float* z, const float* mask, const void* packed, float* out,
                       int add_residual, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_z,
                       int c_hidden, uint32_t* status, void* stream) {
  return trimul_forward_impl(outgoing, z, mask, packed, out, add_residual, DropArgs{}, workspace, workspace_bytes, B,
                             N, c_z, c_hidden, status, stream);
}

int gtk_trimul_forward_dropout(int outgoing, const float* z, const float* mask, const void* packed, float* out,
                               int add_residual, const gtk_dropout* dropout, void* workspace, size_t workspace_bytes,
                               int64_t B, int64_t N, int c_z, int c_hidden, uint32_t* status, void* stream) {
  DropArgs d{};
  // The update's pair frame is z's own: DropoutRowwise's vector is the column j.
  if (int e = drop_args(dropout, B, N, /*transposed=*/false, c_z, &d)) return e;
  return trimul_forward_impl(outgoing, z, mask, packed, out, add_residual, d, workspace, workspace_bytes, B, N, c_z,
                             c_hidden, status, stream);
}

int gtk_trimul_forward_noalloc(int outgoing, const float* z, const float* mask, const void* packed, float* out,
                               int add_residual, int64_t B, int64_t N, int c_z, int c_hidden, uint32_t* status,
                               void* stream) {
  if (c_z != 128 || c_hidden != 128)
    return fail(GTK_ERR_UNSUPPORTED, "trimul: only c_z = c_hidden = 128 is implemented");
  if (!dims_ok(B, 65535) || !dims_ok(N, 65535)) return fail(GTK_ERR_INVALID_ARG, "trimul: bad B/N");
  const size_t need = gtk_trimul_workspace_bytes(B, N, c_z, c_hidden);
  if (need > kNoAllocScratchBytes)
    return fail(GTK_ERR_WORKSPACE, "trimul_forward_noalloc: B=" + std::to_string(B) + ", N=" + std::to_string(N) +
                                       " needs " + std::to_string(need) + " bytes of scratch; the built-in scratch "
                                       "holds " + std::to_string(kNoAllocScratchBytes) +
                                       " (B * N * round_up(N, 8) <= 32768). Use gtk_trimul_forward with a "
                                       "caller-provided workspace instead.");
  void* scratch = nullptr;
  if (int e = noalloc_scratch_address(&scratch)) return e;
  return gtk_trimul_forward(outgoing, z, mask, packed, out, add_residual, scratch, kNoAllocScratchBytes, B, N, c_z,
                            c_hidden, status, stream);
}

}  // extern "C"
