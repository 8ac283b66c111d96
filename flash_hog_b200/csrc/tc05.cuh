// Blackwell (sm_100a) building blocks: mbarriers with bounded waits, TMA tile
// loads, TMEM allocation and loads, tcgen05.mma issue/commit and the shared
// memory / instruction descriptors the tensor core reads.
//
// Conventions used by every kernel in this library:
//  * bf16 tiles live in shared memory as 128-byte-swizzled "panels": a panel is
//    R rows x 64 bf16 columns (128 bytes per row), rows contiguous, 16-byte
//    chunk c of row r stored at chunk position (c ^ (r % 8)). This is exactly the
//    layout a TMA load with CU_TENSOR_MAP_SWIZZLE_128B and a {64, R} box writes.
//    A tile wider than 64 columns is several panels, each R*128 bytes apart.
//    Panels start on 1024-byte boundaries (the swizzle repeats every 8 rows).
//  * The same panel serves as a K-major operand (K along the 64 columns) or as
//    an MN-major operand (MN along the 64 columns, K along the rows).
//  * TMEM accumulators use cta_group::1, M = 128: TMEM lane i holds row i, column
//    j holds element j. Warp w of a warpgroup may only touch lanes 32*(w%4)...+31.

#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace fh {

// ------------------------------------------------------------------------------------
// status reporting
// ------------------------------------------------------------------------------------

// Error codes a kernel can record in the per-device status word.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutTmaFull = 1,     // waiting for a TMA load to land
  kDevTimeoutSlotEmpty = 2,   // waiting for a ring slot to be released
  kDevTimeoutMma = 3,         // waiting for a tcgen05.commit
  kDevTimeoutEpilogue = 4,    // waiting for the elementwise warps
  kDevTimeoutDrain = 5,       // waiting for in-flight loads during teardown
};

// Upper bound on any single mbarrier wait. Every legitimate wait in these
// kernels is for one pipeline step (microseconds); one second means a lost
// arrival, and the kernel gives up instead of hanging the GPU.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async (TMA / tensor core) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Adds `bytes` to the barrier's expected transaction count without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// One wait attempt: the thread may sleep in the hardware until the phase
// completes or a system-dependent time limit passes, so waiting warps do not
// take issue slots from the warps sharing their scheduler. (An explicit long
// suspend-time hint delayed the wake-up after the phase completed.)
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: true iff the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up (returns
// false) after kWaitLimitNs, or early once another role raised `abort_flag`
// (pass nullptr to ignore the flag, as the teardown drain does).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if (abort_flag && *abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Warp-wide form of mbar_wait: every lane of the warp calls it and all lanes
// leave together as soon as any lane sees the phase complete. Each exit test is
// voted across the warp, so lanes that time out of one try_wait never diverge
// from lanes that saw the phase (a diverged warp waited for its last lane to
// wake). Same limits as mbar_wait.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t a = smem_u32(bar);
  if (__any_sync(0xffffffffu, mbar_try_wait(a, parity))) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (__any_sync(0xffffffffu, mbar_try_wait(a, parity))) return true;
    const bool stop = (abort_flag && *abort_flag) || (global_timer_ns() - t0 > kWaitLimitNs);
    if (__any_sync(0xffffffffu, stop)) return false;
  }
}

// ------------------------------------------------------------------------------------
// TMA
// ------------------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-D tiled load (no multicast) into this CTA's shared memory; completion is
// signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Plain bulk copy global -> shared (both 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tcgen05.mma operands).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------------------
// TMEM
// ------------------------------------------------------------------------------------

// Whole-warp collective. Writes the TMEM base address to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp receives
// lane (base lane + t), columns col .. col+15. Results are valid only after
// tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 8 consecutive 32-bit columns (see tmem_ld16).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns from registers (the store twin of
// tmem_ld16). Visible to tcgen05.mma only after tmem_wait_st().
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Pins register values after tmem_wait_ld(): later uses depend on this empty
// asm, which the compiler keeps after the (volatile) wait.
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// Lane base for the calling warp inside its warpgroup (bits 31:16 of a TMEM address).
__device__ __forceinline__ uint32_t tmem_lane_base(int warp_in_group) {
  return static_cast<uint32_t>(warp_in_group * 32) << 16;
}

// ------------------------------------------------------------------------------------
// tcgen05.mma
// ------------------------------------------------------------------------------------

enum SmemLayout : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

// Shared memory matrix descriptor (Blackwell version 1).
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1)
//   bits 49-51 base offset (0: panels are 1024-byte aligned)   bits 61-63 layout
// K-major, 128B swizzle: SBO = byte distance between 8-row groups (1024 for
//   128-byte rows); LBO unused (encoded as 16 bytes).
// MN-major, 128B swizzle: LBO = byte distance between 64-element MN panels,
//   SBO = byte distance between 8-row K groups (1024).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
         (static_cast<uint64_t>(layout) << 61);
}

// Instruction descriptor for kind::f16 with bf16 A/B and an fp32 accumulator.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format,
//   bit 15 A major (1 = MN), bit 16 B major, bits 17-22 N >> 3, bits 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A * B, issued by a single thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A * B with A read from TMEM: M = 128 lanes, 16 bf16 of K packed
// two per 32-bit column (8 columns per k-step, element k in the low half of
// column k/2 when k is even); B from a shared-memory descriptor.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Warp-convergent forms: the whole warp executes them (descriptors stay
// warp-uniform) and elect.sync picks the one lane that issues.
__device__ __forceinline__ void umma_bf16_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Four chained MMAs into one accumulator from one elected lane (the whole warp
// executes it): one elect.sync and one predicate for the chain instead of per
// instruction, so the issuing warp spends fewer issue slots per MMA.
__device__ __forceinline__ void umma_bf16_x4_w(uint32_t d_tmem, uint64_t a0, uint64_t a1, uint64_t a2, uint64_t a3,
                                               uint64_t b0, uint64_t b1, uint64_t b2, uint64_t b3, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %10, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %9, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %9, 1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %9, 1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %9, 1;\n\t}" ::"r"(d_tmem),
      "l"(a0), "l"(a1), "l"(a2), "l"(a3), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_ts_x4_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0, uint64_t b1,
                                                  uint64_t b2, uint64_t b3, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 t1, t2, t3;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %7, 0;\n\t"
      "add.u32 t1, %1, 8;\n\tadd.u32 t2, %1, 16;\n\tadd.u32 t3, %1, 24;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %6, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], %3, %6, 1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t2], %4, %6, 1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t3], %5, %6, 1;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b0), "l"(b1), "l"(b2), "l"(b3), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_ts_x2_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0, uint64_t b1,
                                                  uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 t1;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "add.u32 t1, %1, 8;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, p;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], %3, %4, 1;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b0), "l"(b1), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------------------------
// operand panels written by threads
// ------------------------------------------------------------------------------------

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128B-swizzled panel.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Hardware base-2 exponential (MUFU.EX2), flushes denormals; exp2(-inf) = 0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Named barrier among `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace fh
