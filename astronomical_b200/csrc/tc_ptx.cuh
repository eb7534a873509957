// tc_ptx.cuh -- thin inline-PTX wrappers for the sm_100a tensor-core path:
// mbarriers (every wait is bounded by a wall-clock deadline), TMA tile loads
// (never with cluster multicast), and the tcgen05 family (TMEM alloc, MMA,
// commit, load, fences).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace astro {
namespace tc {

ASTRO_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

ASTRO_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

ASTRO_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

ASTRO_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

ASTRO_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

ASTRO_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// A waiting thread may be suspended in hardware until the phase completes or
// ASTRO_MBAR_SUSPEND_NS nanoseconds pass (the try_wait suspend-time hint), so
// waiting warps do not take issue slots from the working ones; 0 leaves the
// limit to the system.
#ifndef ASTRO_MBAR_SUSPEND_NS
#define ASTRO_MBAR_SUSPEND_NS 0
#endif
ASTRO_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
#if ASTRO_MBAR_SUSPEND_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(ASTRO_MBAR_SUSPEND_NS)
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

// Bounded wait: returns false after `limit_ns` of waiting (or when another role
// has already raised *abort), having recorded kDevWaitTimeout.
ASTRO_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                            uint32_t* status, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort = 1;
        record_status(status, kDevWaitTimeout);
        return false;
      }
    }
  }
}

// One lane of the (converged, full) warp is elected: true in exactly one lane.
ASTRO_DEVINL bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// 2D TMA tile load global -> shared, completion counted on `bar` (no multicast).
ASTRO_DEVINL void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

ASTRO_DEVINL void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// generic-proxy smem writes -> visible to the async proxy (tcgen05.mma operands)
ASTRO_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 ----
ASTRO_DEVINL void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
ASTRO_DEVINL void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
ASTRO_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
ASTRO_DEVINL void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
ASTRO_DEVINL void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate, M=128.
ASTRO_DEVINL void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: the A operand (M=128 rows in lanes 0..127,
// K packed two bf16 per 32-bit column) is read from tensor memory.
ASTRO_DEVINL void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The four K=16 MMAs of one 64-wide K block in one asm block (the issuing thread
// shares its scheduler with busy warps, so every instruction it saves counts):
// A from TMEM columns a, a+8, a+16, a+24; B descriptors whose low words are
// b_lo, b_lo+2, b_lo+4, b_lo+6 (32-byte steps) with high word b_hi; the first
// MMA accumulates iff acc_first != 0, the rest always do.
ASTRO_DEVINL void mma4_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                               uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b64 b0, b1, b2, b3;\n\t.reg .b32 l1, l2, l3, a1, a2, a3;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "setp.eq.b32 q, %5, %5;\n\t"
      "add.u32 l1, %2, 2;\n\tadd.u32 l2, %2, 4;\n\tadd.u32 l3, %2, 6;\n\t"
      "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
      "mov.b64 b0, {%2, %3};\n\tmov.b64 b1, {l1, %3};\n\t"
      "mov.b64 b2, {l2, %3};\n\tmov.b64 b3, {l3, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b0, %4, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %4, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %4, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %4, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc_first)
      : "memory");
}

// Same with A from shared memory: A descriptors a_lo + 2k, B descriptors b_lo + 2k.
ASTRO_DEVINL void mma4_bf16_ss(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                               uint32_t b_hi, uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b64 a0, a1, a2, a3, b0, b1, b2, b3;\n\t"
      ".reg .b32 x1, x2, x3, y1, y2, y3;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "setp.eq.b32 q, %6, %6;\n\t"
      "add.u32 x1, %1, 2;\n\tadd.u32 x2, %1, 4;\n\tadd.u32 x3, %1, 6;\n\t"
      "add.u32 y1, %3, 2;\n\tadd.u32 y2, %3, 4;\n\tadd.u32 y3, %3, 6;\n\t"
      "mov.b64 a0, {%1, %2};\n\tmov.b64 a1, {x1, %2};\n\t"
      "mov.b64 a2, {x2, %2};\n\tmov.b64 a3, {x3, %2};\n\t"
      "mov.b64 b0, {%3, %4};\n\tmov.b64 b1, {y1, %4};\n\t"
      "mov.b64 b2, {y2, %4};\n\tmov.b64 b3, {y3, %4};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a0, b0, %5, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %5, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %5, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %5, q;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc_first)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i writes lane (base + i).
ASTRO_DEVINL void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
ASTRO_DEVINL void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// arrive on `bar` once every MMA issued so far by this thread has completed
ASTRO_DEVINL void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i receives lane (base + i).
ASTRO_DEVINL void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
ASTRO_DEVINL void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Wait that also ties the destination registers of the outstanding load, so the
// compiler cannot schedule any use of them before the wait.
ASTRO_DEVINL void tmem_ld_wait16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                 "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// Shared-memory matrix descriptor: K-major tile of 128-byte rows with the
// 128-byte swizzle (8-row atoms of 1024 bytes), tile base 1024-byte aligned.
ASTRO_DEVINL uint64_t sdesc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3fffu);       // start address
  d |= (uint64_t)1u << 16;                            // leading byte offset (unused, 16 B)
  d |= (uint64_t)(1024u >> 4) << 32;                  // stride byte offset: 8-row atom
  d |= (uint64_t)1u << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

}  // namespace tc
}  // namespace astro
