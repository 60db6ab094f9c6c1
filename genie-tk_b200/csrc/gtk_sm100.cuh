// Device-side toolkit for the sm_100a kernels of this library: shared-memory
// barriers with bounded waits, TMA bulk-tensor copies, tcgen05 (TMEM + 5th-gen tensor
// core) wrappers and the UMMA shared-memory / instruction descriptors.
//
// Every wait in this file is bounded in wall-clock time (%globaltimer). A wait that
// runs out records a status bit in the caller-provided status word, raises the CTA's
// abort flag and returns false, so the kernel unwinds (drains its copies, frees TMEM)
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gtk {

// ----------------------------------------------------------------------------------
// Status word bits (device side). The host maps a non-zero word to an error code.
// ----------------------------------------------------------------------------------
enum StatusBits : uint32_t {
  kStatusTimeoutProducer = 1u << 0,
  kStatusTimeoutMma = 1u << 1,
  kStatusTimeoutConsumer = 1u << 2,
  kStatusTimeoutDrain = 1u << 3,
  kStatusBadLaunch = 1u << 4,
  kStatusTimeoutPeer = 1u << 5,  // a cross-GPU barrier ran out (a peer never arrived)
  kStatusSaturated = 1u << 6,    // an fp16 intermediate was beyond +-65504 and was clamped
};

// Wall-clock limit for any single wait: 2 s is orders of magnitude above any
// legitimate wait in these kernels.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async proxy (TMA, tcgen05.commit).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Raise the current phase's expected transaction bytes without arriving (a copy split in
// parts: the last part arrives with arrive.expect_tx).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive on `bar` only once `dep` is available. Use it to release a buffer the thread has
// just read with shared-memory loads: pass a value computed from every loaded element. An
// arrive issued right after the loads can complete while some of them are still in flight,
// and a producer that refills the buffer on that signal (a TMA load) would then overwrite
// data not yet read. The opaque zero (IEEE rules keep dep * 0 from being folded; NaN and
// infinities convert to 0) puts a true data dependency between the loads' consumers and
// the arrive.
__device__ __forceinline__ void mbar_arrive_after(uint64_t* bar, float dep) {
  const int zero = __float2int_rz(dep * 0.0f);
  mbar_arrive(reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(bar) + zero));
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA failure state, kept in shared memory.
struct CtaGuard {
  volatile uint32_t abort;  // set when any wait of this CTA ran out
};

// Channel dropout applied by a residual epilogue: one keep vector of `groups` x 128 bits
// per (batch, residue t), channel c at bit c % 32 of word (c % 128) / 32 of its 128-bit group
// c / 128, set when the channel is kept; kept channels are multiplied by `scale`. In a
// kernel's own pair frame (row r, column j) the vector is t = by_row ? r : j, at
// keep[(b * ld + t) * groups].
struct DropArgs {
  const uint4* keep;
  float scale;
  int by_row;
  int groups;
  int64_t ld;
};

// Keep vector of pair (b, r, j) of the kernel frame; all zero (drop) for a column past the
// end of the row (that pair is never stored).
__device__ __forceinline__ uint4 drop_keep(const DropArgs& d, int b, int r, int j, int n_cols) {
  if (!d.by_row && j >= n_cols) return make_uint4(0u, 0u, 0u, 0u);
  return __ldg(d.keep + (static_cast<int64_t>(b) * d.ld + (d.by_row ? r : j)) * d.groups);
}

// Word w of a keep vector (w = 0..3, a runtime index).
__device__ __forceinline__ uint32_t drop_word(const uint4& k, int w) {
  return w == 0 ? k.x : (w == 1 ? k.y : (w == 2 ? k.z : k.w));
}

// Bounded wait on the phase with the given parity. Returns false (after recording
// `code` in *status and raising guard->abort) when the limit passes or when another
// role of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, CtaGuard* guard, uint32_t* status,
                                          uint32_t code) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (guard->abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        guard->abort = 1;
        if (status) atomicOr(status, code);
        return false;
      }
    }
  }
}

// Bounded wait used while unwinding after an abort: ignores the abort flag so that
// copies still in flight land before shared memory is released.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(addr, parity)) {
    if ((++spins & 63u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// ----------------------------------------------------------------------------------
// Proxy fences
// ----------------------------------------------------------------------------------
// Generic-proxy writes to shared memory -> visible to the async proxy (TMA store,
// tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor). Tensor maps are __grid_constant__ kernel parameters.
// Every load and store here moves data between global memory and the issuing CTA alone.
// ----------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, "
      "%6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until the shared-memory sources of all committed stores have been read.
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until at most one committed store group still reads shared memory.
__device__ __forceinline__ void tma_store_wait_read_le1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// Wait until all committed stores are complete (globally performed).
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ----------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads/stores, fences.
// TMEM address: bits [31:16] lane, [15:0] column.
// ----------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on an mbarrier when all previously issued tcgen05 ops of this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 32 consecutive columns: thread t of the warp gets lane (warp%4)*32+t.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 32 bits, 16 consecutive columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// tcgen05.wait::ld that also names the destination registers of the loads it completes, so
// the compiler cannot read, move or copy them before the wait (used when a load is left in
// flight across other work).
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&a)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                 "+r"(a[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&a)[16], uint32_t (&b)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                 "+r"(a[15]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]),
                 "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]),
                 "+r"(b[14]), "+r"(b[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// ----------------------------------------------------------------------------------
// UMMA descriptors (layouts as defined for tcgen05 in the PTX ISA; field positions
// cross-checked against CUTLASS's cute/arch/mma_sm100_desc.hpp).
// ----------------------------------------------------------------------------------
enum class Swz : uint32_t { kNone = 0, k128 = 2, k64 = 4, k32 = 6 };

// Shared-memory matrix descriptor. `lbo`/`sbo` in bytes.
//  K-major, swizzled:  rows of (swizzle width) bytes along K; SBO = byte distance
//                      between consecutive 8-row groups; LBO unused (16).
//  MN-major, swizzled: rows of (swizzle width) bytes along MN, one row per K index;
//                      LBO = byte distance between consecutive MN chunks of one
//                      swizzle width; SBO = byte distance between 8-K-row groups.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, Swz swz) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version for tcgen05
  d |= static_cast<uint64_t>(static_cast<uint32_t>(swz)) << 61;
  return d;
}

// Instruction descriptor, kind::f16 with fp32 accumulator. A and B always share one
// type: fp16 (make_idesc_f16) or bf16 (make_idesc_bf16). a_mn/b_mn: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t make_idesc_16(uint32_t fmt, uint32_t M, uint32_t N, uint32_t a_mn,
                                                     uint32_t b_mn) {
  return (1u << 4)              // D format: f32
         | (fmt << 7)           // A format: 0 = f16, 1 = bf16
         | (fmt << 10)          // B format (same as A)
         | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t M, uint32_t N, uint32_t a_mn, uint32_t b_mn) {
  return make_idesc_16(0u, M, N, a_mn, b_mn);
}
__host__ __device__ constexpr uint32_t make_idesc_bf16(uint32_t M, uint32_t N, uint32_t a_mn, uint32_t b_mn) {
  return make_idesc_16(1u, M, N, a_mn, b_mn);
}

// ----------------------------------------------------------------------------------
// Small numeric helpers
// ----------------------------------------------------------------------------------
// Hardware tanh (one MUFU op); sigmoid(x) = 0.5 * tanh(x / 2) + 0.5.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// fp16 pair with saturation to the finite range (values beyond +-65504 clamp).
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  lo = fminf(fmaxf(lo, -65504.f), 65504.f);
  hi = fminf(fmaxf(hi, -65504.f), 65504.f);
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ __half f16_sat(float x) { return __float2half_rn(fminf(fmaxf(x, -65504.f), 65504.f)); }

// The same conversions for values that are not bounded by construction: `sat` records
// whether either input was beyond the fp16 range (and so was clamped).
__device__ __forceinline__ uint32_t pack_f16x2_chk(float lo, float hi, uint32_t& sat) {
  sat |= static_cast<uint32_t>(fmaxf(fabsf(lo), fabsf(hi)) > 65504.f);
  return pack_f16x2(lo, hi);
}
__device__ __forceinline__ __half f16_sat_chk(float x, uint32_t& sat) {
  sat |= static_cast<uint32_t>(fabsf(x) > 65504.f);
  return f16_sat(x);
}
// Report a clamp seen by this thread in the caller's status word (GTK_STATUS_FP16_SATURATED).
__device__ __forceinline__ void flag_saturation(uint32_t sat, uint32_t* status) {
  if (sat && status) atomicOr(status, kStatusSaturated);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled tile
// whose rows are 128 bytes (the TMA SWIZZLE_128B pattern; tile base 1024-B aligned).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ----------------------------------------------------------------------------------
// Shared-memory helpers used by several kernels
// ----------------------------------------------------------------------------------
__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t a = smem_u32(p);
  return p + (((a + 1023u) & ~1023u) - a);
}

__device__ __forceinline__ float4 lds_f4(const uint8_t* p) { return *reinterpret_cast<const float4*>(p); }
// 32-byte global store (sm_100); p must be 32-byte aligned.
__device__ __forceinline__ void stg_v8(void* p, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t a4,
                                       uint32_t a5, uint32_t a6, uint32_t a7) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a0), "r"(a1), "r"(a2),
               "r"(a3), "r"(a4), "r"(a5), "r"(a6), "r"(a7)
               : "memory");
}
__device__ __forceinline__ void sts_u4(uint8_t* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

}  // namespace gtk
