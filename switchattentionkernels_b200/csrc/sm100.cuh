// Blackwell (sm_100a) building blocks used by the Switch Attention kernels:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM allocation,
// UMMA issue, commit, TMEM load/store) and shared-memory matrix descriptors.
//
// Everything here is hand-written inline PTX.  Descriptor bit layouts follow the
// PTX ISA "matrix descriptor" and "instruction descriptor" tables for
// tcgen05.mma (kind::f16); they were cross-checked against the public CUTLASS
// headers (cute/arch/mma_sm100_desc.hpp).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace swa {

// ---------------------------------------------------------------------------
// generic helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait on an mbarrier is bounded.  A wait that exceeds kWaitLimitNs sets
// the CTA-wide abort flag (shared memory) and returns false; every other wait
// sees the flag and returns false as well, so all roles leave their loops, the
// CTA frees its tensor memory and the kernel returns with an error code recorded
// in global memory.  No legitimate wait in these kernels lasts longer than one
// work unit (well under 10 ms), so one second is a wide margin.  Named barriers
// (bar.sync) have no time limit, so a kernel that uses one (the decode step's
// four math warps) places it where every warp arrives whether or not it left its
// loop on an abort; the prefill kernel uses none.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false when the CTA
// is aborting (the flag was set here or by another role).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled, no multicast: every CTA issues its own loads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// The same tile loads with an L2 cache policy (createpolicy) for the lines they read.
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, int c3, int c4, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "l"(policy)
      : "memory");
}

// L2 policy for data read or written once (evict-first).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 16-byte global store with an L2 cache policy.
__device__ __forceinline__ void st_global_v4_hint(void* ptr, uint4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(ptr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w), "l"(policy)
               : "memory");
}

// L2 policy that keeps lines resident ahead of streaming data (evict-last).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory
// ---------------------------------------------------------------------------
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

// Make this thread's generic-proxy writes to shared memory (st.shared,
// cp.async) visible to later async-proxy reads (tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Warp-converged issue: the whole warp executes these calls (descriptors stay warp
// uniform) and one lane chosen by elect.sync issues the tcgen05 instructions.
// Issuing tcgen05.mma from a single lane inside a divergent branch measured 2-3x
// the MMA's own duration; converged issue runs at the tensor peak.
//
// Arrive (once) on `bar` when every tcgen05 operation issued so far by the
// elected thread has completed.
__device__ __forceinline__ void tc_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Eight back-to-back SS MMAs over K = 128 with all sixteen descriptors given in
// registers (a[k], b[k]: step k's operands), so the first MMA issues right after
// the elect and the issuing warp does no address arithmetic on the critical path.
// The first step overwrites D.
__device__ __forceinline__ void umma_ss8_warp(uint32_t d_tmem, const uint64_t* a, const uint64_t* b, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, p0, p1;\n\t"
      "setp.ne.b32 p0, 0, 0;\n\tsetp.eq.b32 p1, 0, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %9, %17, p0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %10, %17, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %11, %17, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %12, %17, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %13, %17, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %14, %17, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %15, %17, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %16, %17, p1;\n\t}" ::"r"(d_tmem),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]),
      "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "r"(idesc)
      : "memory");
}

// Start-address offsets (descriptor units of 16 bytes) of the eight K = 16 steps of a
// 128-column K-major tile stored as two 64-column swizzled halves 16 KB apart.
__host__ __device__ constexpr uint32_t k128_step_offset(int k) { return (k >> 2) * 1024 + (k & 3) * 2; }

// As umma_ss_k128_warp with an N = 64 B operand whose two 64-column halves lie
// 8192 bytes apart (a 64-row swizzled tile); A's halves lie 16384 bytes apart.
__device__ __forceinline__ void umma_ss_k128_bhalf8k_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                          uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, p0, p1;\n\t.reg .b64 a1, a2, a3, a4, a5, a6, a7, b1, b2, b3, b4, b5, b6, b7;\n\t"
      "setp.ne.b32 p0, 0, 0;\n\tsetp.eq.b32 p1, 0, 0;\n\t"
      "add.s64 a1, %1, 2;\n\tadd.s64 a2, %1, 4;\n\tadd.s64 a3, %1, 6;\n\tadd.s64 a4, %1, 1024;\n\t"
      "add.s64 a5, %1, 1026;\n\tadd.s64 a6, %1, 1028;\n\tadd.s64 a7, %1, 1030;\n\t"
      "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\tadd.s64 b4, %2, 512;\n\t"
      "add.s64 b5, %2, 514;\n\tadd.s64 b6, %2, 516;\n\tadd.s64 b7, %2, 518;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a4, b4, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a5, b5, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a6, b6, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a7, b7, %3, p1;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}

// Two back-to-back TS MMAs over 32 keys (A = P from TMEM, 8 columns per 16 keys;
// B = V MN-major, 2048 bytes per 16 keys); `accumulate_first` = 0 makes the first
// step overwrite D.
__device__ __forceinline__ void umma_ts_k32_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate_first) {
  asm volatile(
      "{\n\t.reg .pred e, pf, p1;\n\t.reg .b64 b1;\n\t.reg .b32 t1;\n\t"
      "setp.ne.b32 pf, %4, 0;\n\tsetp.eq.b32 p1, 0, 0;\n\t"
      "add.s64 b1, %2, 128;\n\tadd.u32 t1, %1, 8;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pf;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], b1, %3, p1;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate_first)
      : "memory");
}

// Eight back-to-back TS MMAs over K = 128: A (M x 128, BF16 pairs) from TMEM, 8
// columns per 16-element step; B a K-major 64-row swizzled tile whose two
// 64-column halves lie 8192 bytes apart (step kk adds (kk / 4) * 8192 +
// (kk % 4) * 32 bytes to its start address).  The first step overwrites D.
__device__ __forceinline__ void umma_ts_k128_bhalf8k_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                          uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, p0, p1;\n\t.reg .b64 b1, b2, b3, b4, b5, b6, b7;\n\t"
      ".reg .b32 a1, a2, a3, a4, a5, a6, a7;\n\t"
      "setp.ne.b32 p0, 0, 0;\n\tsetp.eq.b32 p1, 0, 0;\n\t"
      "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\tadd.u32 a4, %1, 32;\n\t"
      "add.u32 a5, %1, 40;\n\tadd.u32 a6, %1, 48;\n\tadd.u32 a7, %1, 56;\n\t"
      "add.s64 b1, %2, 2;\n\tadd.s64 b2, %2, 4;\n\tadd.s64 b3, %2, 6;\n\tadd.s64 b4, %2, 512;\n\t"
      "add.s64 b5, %2, 514;\n\tadd.s64 b6, %2, 516;\n\tadd.s64 b7, %2, 518;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a4], b4, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a5], b5, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a6], b6, %3, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a7], b7, %3, p1;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc)
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm100 version field = 1.
//   K-major operand : lbo ignored (pass 16), sbo = byte stride between 8-row groups.
//   MN-major operand: lbo = byte stride between 64-element MN blocks,
//                     sbo = byte stride between 8-row K groups.
__device__ __forceinline__ uint64_t make_smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;  // descriptor version (sm100)
  d |= static_cast<uint64_t>(2u) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with BF16 A/B and FP32 accumulation.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                   // D format: F32
         | (1u << 7)                                 // A format: BF16
         | (1u << 10)                                // B format: BF16
         | ((a_mn_major ? 1u : 0u) << 15)            // A major
         | ((b_mn_major ? 1u : 0u) << 16)            // B major
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM <-> registers (32 lanes x 32-bit, 32 consecutive columns)
// ---------------------------------------------------------------------------
#define SWA_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                  "=r"(r[i + 6]), "=r"(r[i + 7])
#define SWA_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                  "r"(r[i + 6]), "r"(r[i + 7])

__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : SWA_R8(0), SWA_R8(8), SWA_R8(16), SWA_R8(24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : SWA_R8(0), SWA_R8(8)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      SWA_W8(0), SWA_W8(8)
      : "memory");
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      SWA_W8(0), SWA_W8(8), SWA_W8(16), SWA_W8(24)
      : "memory");
}

__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), SWA_W8(0)
               : "memory");
}

// 16-lane forms (".16x32bx2"): the warp accesses 16 TMEM lanes (the lane field of
// taddr: its quarter's lane 0 or 16); threads 0-15 get columns [c, c + n) of lanes
// 0..15, threads 16-31 columns [c + n, c + 2n) of the same lanes (second access at
// the immediate column offset n).  So the two threads t and t + 16 of a warp share
// one row and hold adjacent column ranges of it.
__device__ __forceinline__ void tmem_ld_16x2_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32], 32;"
      : SWA_R8(0), SWA_R8(8), SWA_R8(16), SWA_R8(24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_16x2_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16], 16;"
      : SWA_R8(0), SWA_R8(8)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_16x2_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], 16, "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      SWA_W8(0), SWA_W8(8)
      : "memory");
}

#undef SWA_R8
#undef SWA_W8

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Register fence: ties the 32 registers to this point in program order so that no
// use of a tcgen05.ld result is scheduled before the tcgen05.wait::ld above it.
__device__ __forceinline__ void reg_fence32(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

// Named barrier over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void reg_fence16(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(r[i]));
}

// ---------------------------------------------------------------------------
// math helpers (hardware instructions only)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// x if (mask & bit) != 0, else -inf, as a predicated select: no branch, since the
// masks of the lanes of a warp differ.
__device__ __forceinline__ float select_or_neg_inf(uint32_t mask, uint32_t bit, float x) {
  float y;
  asm("{\n\t.reg .pred p;\n\t.reg .b32 t;\n\t"
      "and.b32 t, %1, %2;\n\t"
      "setp.ne.b32 p, t, 0;\n\t"
      "selp.f32 %0, %3, 0fFF800000, p;\n\t}"
      : "=f"(y)
      : "r"(mask), "r"(bit), "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed FP32 pairs (sm_100 f32x2 instructions); lo = first element.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}

__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  // cvt packs its first source into the upper half.
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

}  // namespace swa
