// PTX wrappers for a pair of CTAs (a cluster of 2 on neighbouring SMs) driving one
// cta_group::2 tcgen05 MMA: M = 256 rows, 128 in each CTA's tensor memory; each CTA holds
// half of the B operand's N extent in its own shared memory. No multicast loads: every CTA
// loads its own operand halves; only MMA completion is signalled to both CTAs at once
// (tcgen05.commit with a CTA mask).
#pragma once

#include <stdint.h>

#include "sm100_ptx.cuh"

namespace ta {

__device__ __forceinline__ uint32_t cluster_cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the object at `local` (this CTA's shared memory) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

// Arrive on an mbarrier of either CTA of the pair, given by its shared::cluster address,
// with release semantics at cluster scope: orders this thread's prior shared-memory accesses
// (e.g. stores into the other CTA) before the arrival. Measured ~3000 clocks from the other
// SM, so used only once per work item.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Plain remote arrive (default semantics), for hand-offs of tensor-memory data: the writer's
// tcgen05.wait + tcgen05.fence::before_thread_sync and the reader's
// tcgen05.fence::after_thread_sync order the tensor-memory accesses themselves (the form
// CUTLASS's cluster barriers use). Lands in the other SM within ~100s of clocks.
__device__ __forceinline__ void mbar_arrive_cluster_tc(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 32-bit store into another CTA's shared memory (shared::cluster address).
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// Non-suspending phase test with acquire at cluster scope, for barriers that receive
// arrivals from the peer CTA: a thread suspended in try_wait was measured to wake up late
// (~3000 clocks) when the completing arrival came from the other SM, so these are polled.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait (same contract as mbar_wait_bounded) with cluster-scope acquire.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity,
                                                          volatile int* abort_flag,
                                                          uint64_t timeout_ns) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait_cluster(a, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(a, parity)) return true;
    if ((it & 255u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > timeout_ns) return false;
    }
  }
}

// All threads of both CTAs (hardware cluster barrier; every path of the kernel reaches it).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// Tensor memory for a CTA pair: executed by the same warp in both CTAs.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem, both CTAs] (+)= A[smem, both CTAs] * B[smem, both CTAs], M = 256 (issued by the
// even CTA of the pair).
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem], both CTAs, M = 256.
__device__ __forceinline__ void mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask` when all async
// tcgen05 operations issued so far by this thread (pair MMAs) are complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// 4-D tiled bulk tensor load into this CTA's shared memory whose completion (bytes) is
// counted on an mbarrier of either CTA of the pair (shared::cluster address). No multicast.
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster_addr, int c0, int c1,
                                                 int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

}  // namespace ta
