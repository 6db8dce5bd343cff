// 5th-generation tensor core (tcgen05 / TMEM) and TMA primitives shared by the GEMM and attention kernels (sm_100a).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace svx {
namespace tc {

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// TMA store of a shared-memory box to global memory (bulk async-group completion), one thread.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until this thread's committed bulk stores are complete (visible in global memory).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Warp-collective forms (all 32 lanes call them converged; one elected lane performs the operation). Keeping the
// issue loop warp-uniform lets the compiler hold descriptors and coordinates in uniform registers, which the tensor
// core and TMA instructions take directly; issuing from a single divergent lane costs ~100 cycles per instruction.
__device__ __forceinline__ void tma_load_3d_w(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                              uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      "\n\t}"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void expect_tx_w(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_addr(bar)), "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// UMMA shared-memory descriptor (sm_100 version bit), swizzled canonical layouts. K-major: 8-row atoms whose rows are
// the swizzle width (128 or 64 B), atoms `sbo` bytes apart, LBO unused. MN-major: rows of one swizzle width along MN,
// 8 K-rows per atom `sbo` bytes apart, atoms along MN `lbo` bytes apart. Layout field: 2 = 128B swizzle, 4 = 64B.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes = 16, uint32_t sbo_bytes = 1024) {
  return smem_desc(saddr, lbo_bytes, sbo_bytes, 2);
}
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr, uint32_t lbo_bytes = 16, uint32_t sbo_bytes = 512) {
  return smem_desc(saddr, lbo_bytes, sbo_bytes, 4);
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, A K-major, B K-major (b_mn = false) or MN-major.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool b_mn = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

// Batched issue for attention tiles (warp-collective, one elect for the whole batch; descriptors advance by
// constants, so the issuing warp spends a few instructions per product).
// S = Q K^T over K = 96: four K-steps in the 128B-swizzled parts (qw, kw), two in the 64B-swizzled parts (qn, kn);
// each K-step advances the start address by 32 bytes (+2 in descriptor units).
__device__ __forceinline__ void mma_qk96_w(uint32_t d, uint64_t qw, uint64_t kw, uint64_t qn, uint64_t kn,
                                           uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 a, b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, %5, %5;\n\tsetp.eq.b32 pt, %5, %5;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %5, pf;\n\t"
      "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %5, pt;\n\t"
      "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %5, pt;\n\t"
      "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %5, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %4, %5, pt;\n\t"
      "add.s64 a, %3, 2;\n\tadd.s64 b, %4, 2;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %5, pt;\n\t}"
      ::"r"(d), "l"(qw), "l"(kw), "l"(qn), "l"(kn), "r"(idesc));
}

// O += P V over K = 96 keys: A = P in TMEM (8 columns per K-step; steps 0-3 at `a_lo`, steps 4-5 at `a_hi`), B = V
// MN-major 128B-swizzled (16 keys x 128 B = 2048 bytes per K-step, +128 in descriptor units).
__device__ __forceinline__ void mma_pv96_w(uint32_t d, uint32_t a_lo, uint32_t a_hi, uint64_t v, uint32_t idesc,
                                           uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred e, p0, pt;\n\t.reg .b64 b;\n\t.reg .b32 t;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p0, %5, 0;\n\tsetp.eq.b32 pt, %4, %4;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %4, p0;\n\t"
      "add.s32 t, %1, 8;\n\tadd.s64 b, %3, 128;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t], b, %4, pt;\n\t"
      "add.s32 t, %1, 16;\n\tadd.s64 b, %3, 256;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t], b, %4, pt;\n\t"
      "add.s32 t, %1, 24;\n\tadd.s64 b, %3, 384;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t], b, %4, pt;\n\t"
      "add.s64 b, %3, 512;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], b, %4, pt;\n\t"
      "add.s32 t, %2, 8;\n\tadd.s64 b, %3, 640;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [t], b, %4, pt;\n\t}"
      ::"r"(d), "r"(a_lo), "r"(a_hi), "l"(v), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void commit_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
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

__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x on the special-function unit (max relative error ~2^-22; x = -inf gives 0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two fp32 values rounded to nearest-even bf16 and packed (lo in bits 0-15).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(d) : "f"(lo), "f"(hi));
  return d;
}

__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA, tensor cores).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(columns));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t tmem, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(columns));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait that also gives up as soon as another role of the CTA raised `abort`.
__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (global_timer_ns() - start > kWaitNanoseconds) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2): the even CTA issues M=256 products over both SMs.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory object in CTA `rank` of the cluster (shared::cluster window).
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}

// TMA load into this CTA's shared memory whose completion is counted on an mbarrier of either CTA of the pair
// (`bar` in the shared::cluster window). Warp-collective, one elected lane issues; no multicast.
__device__ __forceinline__ void tma_load_2d_pair_w(void* dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n\t}"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_pair_w(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

// Arrive (once) on the mbarrier at this offset in every CTA of `mask` when the pair's prior products complete.
__device__ __forceinline__ void commit_pair_w(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}"
      ::"r"(smem_addr(bar)), "h"(mask)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(columns));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t tmem, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(columns));
}

// Arrive on an mbarrier of a CTA of this cluster (address in the shared::cluster window).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Warp-collective bounded wait: every lane polls; the warp agrees on the outcome (and is converged afterwards).
__device__ __forceinline__ bool wait_w(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
  return __all_sync(0xffffffffu, wait(bar, parity, abort));
}

}  // namespace tc
}  // namespace svx
