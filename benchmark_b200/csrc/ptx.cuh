// Blackwell (sm_100a) PTX primitives used by the attention and GEMM kernels.
//
// Plays the role of the reference's 0.attention/ptx_wrappers.cuh (mbarrier,
// TMA, tcgen05 alloc/mma/commit/ld/st, descriptors), written for this build:
//   * every mbarrier wait is bounded (globaltimer) and reports a timeout in a
//     device-global status word instead of spinning forever;
//   * no TMA multicast form exists in this file: every load is issued by the
//     CTA that consumes it;
//   * descriptors are built from the tcgen05 shared-memory descriptor and
//     instruction-descriptor bit layouts (PTX ISA, "tcgen05 matrix descriptors").
#pragma once

#include <cstdint>
#include <cuda.h>  // CUtensorMap (type only; the driver is reached via cudaGetDriverEntryPoint)

namespace b200 {

// ---------------------------------------------------------------------------
// Device-global status word.  Bit 0: a bounded wait ran out.  Bits 8..15: the
// wait site that first gave up.  Read and cleared by b200_check().
// ---------------------------------------------------------------------------
// Defined here because the library is built as one translation unit.
__device__ uint32_t g_status = 0;

constexpr uint32_t kStatusTimeout = 1u;
// A pipeline wait inside one CTA never legitimately takes more than a few
// milliseconds; one second separates "slow" from "will never arrive".
constexpr uint64_t kDefaultWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// One arrival for the whole (converged) warp: an elected lane arrives, with no
// divergent branch around it.
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e mbarrier.arrive.shared::cta.b64 _, [%0];\n}\n" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Non-blocking check of a phase (acquire semantics at CTA scope).  A
// test_wait whose result is branched on stalls the thread for its latency
// (hundreds of cycles on B200), so hot waits poll several barriers at once
// (mbar_test3) and keep their slow loop out of line.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Blocking variant: the thread may sleep inside the instruction (up to
// hint_ns) until the phase completes, so waiting warps stop competing for
// issue slots with the warps that share their scheduler.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar_addr, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Record a timeout (first site wins) and return.  Never traps.
__device__ __forceinline__ void report_timeout(uint32_t site) {
  atomicCAS(&g_status, 0u, kStatusTimeout | ((site & 0xffu) << 8));
}

__device__ __forceinline__ bool mbar_wait_slow(uint32_t addr, uint32_t parity, uint32_t site,
                                            uint64_t limit_ns, uint32_t sleep_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (sleep_ns ? mbar_try_wait_sleep(addr, parity, sleep_ns) : mbar_try_wait(addr, parity))
      return true;
    if ((it & 31u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(&g_status) != 0u) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        report_timeout(site);
        return false;
      }
    }
  }
}

// Wait until the phase with the given parity has completed.  Returns false if
// the limit ran out or another wait anywhere on the device already gave up;
// callers then unwind without issuing further dependent work.  sleep_ns > 0
// lets the thread sleep in the hardware wait between polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t site,
                                          uint64_t limit_ns = kDefaultWaitLimitNs,
                                          uint32_t sleep_ns = 0) {
  const uint32_t addr = smem_u32(bar);
  return mbar_try_wait(addr, parity) || mbar_wait_slow(addr, parity, site, limit_ns, sleep_ns);
}

// Poll three barriers in one instruction group: the test_waits do not depend
// on each other, so their latencies overlap instead of adding up.  Pass an
// already-completed (barrier, parity) to fill unused slots.
__device__ __forceinline__ bool mbar_test3(uint32_t a0, uint32_t p0, uint32_t a1, uint32_t p1,
                                           uint32_t a2, uint32_t p2) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred q0, q1, q2;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 q0, [%1], %2;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 q1, [%3], %4;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 q2, [%5], %6;\n"
      " and.pred q0, q0, q1;\n and.pred q0, q0, q2;\n"
      " selp.u32 %0, 1, 0, q0;\n}\n"
      : "=r"(ok)
      : "r"(a0), "r"(p0), "r"(a1), "r"(p1), "r"(a2), "r"(p2)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait3_slow(uint32_t a0, uint32_t p0, uint32_t a1, uint32_t p1,
                                             uint32_t a2, uint32_t p2, uint32_t site) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(a0, p0, 20000u) && mbar_try_wait_sleep(a1, p1, 20000u) &&
        mbar_try_wait_sleep(a2, p2, 20000u))
      return true;
    if ((it & 31u) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(&g_status) != 0u) return false;
      if (globaltimer_ns() - t0 > kDefaultWaitLimitNs) {
        report_timeout(site);
        return false;
      }
    }
  }
}

// Bounded wait for three phases at once (fast path inline, loop out of line).
__device__ __forceinline__ bool mbar_wait3(uint32_t a0, uint32_t p0, uint32_t a1, uint32_t p1,
                                           uint32_t a2, uint32_t p2, uint32_t site) {
  return mbar_test3(a0, p0, a1, p1, a2, p2) || mbar_wait3_slow(a0, p0, a1, p1, a2, p2, site);
}

// ---------------------------------------------------------------------------
// Named barriers (ids 1..15; 0 is __syncthreads)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Per-warpgroup register re-balancing.  Every warp of a warpgroup executes
// the same instruction.  An increase waits until the block's pool (threads x
// registers per thread at launch) has the registers, so the caller must make
// the warpgroups' new counts sum to exactly that pool.
// ---------------------------------------------------------------------------
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor copies).  No multicast variants exist in this build.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x,
                                             int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x,
                                             int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 2-D tile store with an L2 eviction-priority hint (a createpolicy value).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, const void* src, int x,
                                                  int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint"
      " [%0, {%2, %3}], [%1], %4;" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// The same store with an L2 eviction-priority hint (a createpolicy value).
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* map, const void* src, int x,
                                                  int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group.L2::cache_hint"
      " [%0, {%2, %3, %4}], [%1], %5;" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Generic-proxy shared-memory writes become visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ---------------------------------------------------------------------------
// Whole-warp instruction.  Writes the TMEM base address to *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: MMA (kind::f16, bf16 inputs, fp32 accumulate), single issuing thread
// ---------------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-converged issue: the whole warp executes these with the same operands
// (so descriptors stay in uniform registers) and one elected lane issues.
__device__ __forceinline__ void mma_ss_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Arrive (once) on a CTA-local mbarrier when every tcgen05 operation this
// thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2, tcgen05 cta_group::2)
//
// The even CTA of a pair issues the MMAs; each MMA reads A (M/2 rows) and B
// (N/2 rows) from the same shared-memory offset in both CTAs and writes the
// accumulator rows of each CTA into that CTA's TMEM.  A kernel that uses any
// of these uses cta_group::2 for every tcgen05 allocation, MMA and commit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the object at local shared address `addr` in
// the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Whole-cluster barrier; every thread of every CTA of the cluster executes it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier that may live in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   cluster_addr)
               : "memory");
}

// TMA 2D load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (`bar_cluster` from mapa_shared).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::"
      "bytes.L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
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

__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// When every pair MMA this thread issued so far has completed, arrive once on
// the mbarrier at the same shared offset in each CTA named in cta_mask.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Warp-converged forms: the whole warp executes them with the same operands
// and one elected lane issues.
__device__ __forceinline__ void mma_ss_pair_warp(uint32_t d_tmem, uint64_t a_desc,
                                                 uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit_pair_both_warp(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;\n}\n" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Same, for an mbarrier of the issuing CTA only.
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_commit_pair_local_warp(uint64_t* bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Pair MMA with A in TMEM: each CTA supplies its M/2 rows of A from its own
// TMEM at a_tmem, and its N/2 rows of B from shared memory.
__device__ __forceinline__ void mma_ts_pair_warp(uint32_t d_tmem, uint32_t a_tmem,
                                                 uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p, e;\n setp.ne.b32 p, %4, 0;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// TMA 3D load into this CTA's shared memory counted on an mbarrier of either
// CTA of the pair (`bar_cluster` from mapa_shared); no multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int x, int y, int z,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::"
      "bytes.L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z),
      "l"(policy)
      : "memory");
}

// Sleep for about `ns` nanoseconds (unwinding only: lets copies this CTA
// issued land on barriers it cannot observe).
__device__ __forceinline__ void spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) __nanosleep(1000);
}

// Arrive once per warp (elected lane) on an mbarrier that may live in the
// other CTA of the cluster, with the default (release, CTA-scope) semantics:
// what it publishes is TMEM written by tcgen05.st and completed by
// tcgen05.wait::st + tcgen05.fence::before_thread_sync, which the pair's MMAs
// read; a cluster-scope release costs about 1,100 cycles per arrive here.
__device__ __forceinline__ void mbar_arrive_cluster_warp(uint32_t cluster_addr) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e mbarrier.arrive.shared::cluster.b64 _, [%0];\n}\n" ::"r"(cluster_addr)
      : "memory");
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Instruction descriptor, kind::f16: fp32 D, bf16 A and B.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format,
//   15 A major (1 = MN), 16 B major (1 = MN), 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((static_cast<uint32_t>(N) >> 3) << 17) |
         ((static_cast<uint32_t>(M) >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2 in bits
// 61-63), descriptor version 1 (bit 46).  Addresses and offsets in bytes.
//   K-major:  8-row x 128-byte swizzle atoms stacked along M/N at SBO bytes;
//             LBO unused (encoded as 1).  K steps of 16 bf16 advance the start
//             address by 32 bytes inside the atom.
//   MN-major: 64-element x 8-row atoms; LBO = byte distance between 64-element
//             blocks along M/N, SBO = distance between 8-row groups along K.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3fffu) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3fffu) << 32) |
         (static_cast<uint64_t>(1u) << 46) | (static_cast<uint64_t>(2u) << 61);
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM <-> registers.  32x32b shape: thread i of the warp accesses
// TMEM lane (32 * (warp % 4) + i); consecutive registers are consecutive
// 32-bit columns.
// ---------------------------------------------------------------------------
#define B200_R8(a, o) \
  "=r"(a[o + 0]), "=r"(a[o + 1]), "=r"(a[o + 2]), "=r"(a[o + 3]), "=r"(a[o + 4]), \
      "=r"(a[o + 5]), "=r"(a[o + 6]), "=r"(a[o + 7])
#define B200_W8(a, o) \
  "r"(a[o + 0]), "r"(a[o + 1]), "r"(a[o + 2]), "r"(a[o + 3]), "r"(a[o + 4]), "r"(a[o + 5]), \
      "r"(a[o + 6]), "r"(a[o + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : B200_R8(r, 0), B200_R8(r, 8), B200_R8(r, 16), B200_R8(r, 24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : B200_R8(r, 0), B200_R8(r, 8), B200_R8(r, 16), B200_R8(r, 24), B200_R8(r, 32),
        B200_R8(r, 40), B200_R8(r, 48), B200_R8(r, 56)
      : "r"(taddr));
}

// 16-lane shapes: a warp reads or writes 16 TMEM lanes (rows) starting at
// the lane in taddr (0 or 16 within its 32-lane sub-partition).
//   16x256b.xN (ld): thread t holds rows t/4 and t/4+8, columns 8k+2(t%4) and
//                    8k+2(t%4)+1 of every repeat k: r[4k+0] (row t/4, col
//                    8k+2(t%4)), r[4k+1] (same row, next col), r[4k+2] and
//                    r[4k+3] (row t/4+8, the same two cols).
//   16x128b.xN (st): thread t holds column 4k+(t%4) of rows t/4 (r[2k]) and
//                    t/4+8 (r[2k+1]).
__device__ __forceinline__ void tmem_ld_16x256b_x16(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : B200_R8(r, 0), B200_R8(r, 8), B200_R8(r, 16), B200_R8(r, 24), B200_R8(r, 32),
        B200_R8(r, 40), B200_R8(r, 48), B200_R8(r, 56)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : B200_R8(r, 0), B200_R8(r, 8), B200_R8(r, 16), B200_R8(r, 24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_16x256b_x8(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      B200_W8(r, 0), B200_W8(r, 8), B200_W8(r, 16), B200_W8(r, 24)
      : "memory");
}

__device__ __forceinline__ void tmem_st_16x128b_x8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      B200_W8(r, 0), B200_W8(r, 8)
      : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : B200_R8(r, 0)
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : B200_R8(r, 0), B200_R8(r, 8)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      B200_W8(r, 0), B200_W8(r, 8), B200_W8(r, 16), B200_W8(r, 24)
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
          taddr),
      B200_W8(r, 0)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      B200_W8(r, 0), B200_W8(r, 8)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Waits for this thread's outstanding tcgen05.ld and marks the 32 given
// registers as written here, so the compiler cannot move any use of them
// above the wait.
#define B200_RW8(a, o)                                                                   \
  "+r"(a[o + 0]), "+r"(a[o + 1]), "+r"(a[o + 2]), "+r"(a[o + 3]), "+r"(a[o + 4]), \
      "+r"(a[o + 5]), "+r"(a[o + 6]), "+r"(a[o + 7])
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : B200_RW8(r, 0), B200_RW8(r, 8), B200_RW8(r, 16), B200_RW8(r, 24)
               :
               : "memory");
}

// No instruction: marks the 32 registers as written here.  Placed after a
// tcgen05.wait::ld that covers their load, it keeps the compiler from moving
// any use of them above that wait.
__device__ __forceinline__ void reg_written_here(uint32_t (&r)[32]) {
  asm volatile("" : B200_RW8(r, 0), B200_RW8(r, 8), B200_RW8(r, 16), B200_RW8(r, 24));
}

__device__ __forceinline__ void reg_written_here8(uint32_t (&r)[8]) {
  asm volatile("" : B200_RW8(r, 0));
}

__device__ __forceinline__ void reg_written_here16(uint32_t (&r)[16]) {
  asm volatile("" : B200_RW8(r, 0), B200_RW8(r, 8));
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Math helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^e for an integer-valued e (or -inf), built in the exponent field: exact,
// 0 below 2^-126 (and for -inf), +inf above 2^127.
__device__ __forceinline__ float exp2i(float e) {
  if (e < -126.0f) return 0.0f;
  if (e > 127.0f) return __int_as_float(0x7f800000);
  return __int_as_float((static_cast<int>(e) + 127) << 23);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): lo in bits 0-31.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
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

__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// exp2 of two values on the FMA pipe (inputs clamped to [-125, 126]):
//   x = j + r with j = round(x) (adding 1.5 * 2^23 leaves round(x) in the low
//   mantissa bits of t), r in [-0.5, 0.5];  2^r ~ c0 + r(c1 + r(c2 + r c3)),
//   a degree-3 minimax fit of the relative error (7.5e-5) produced by
//   benchmark_b200/csrc/fit_exp2_poly.py;  2^j is applied by adding j << 23
//   to the exponent field (t's bit pattern << 23 is exactly j << 23).
// The clamp keeps the exponent field normal: with j >= -125 and p >= 2^-0.5
// the sum never reaches the subnormal range (at j = -126 a p just below 1
// would), and j <= 126 never overflows.  So x < -125 gives 2^-125 (MUFU's
// ftz form gives 0 below 2^-126) and x > 126 gives 2^126.
__device__ __forceinline__ void exp2_fma_x2(float x0, float x1, float& y0, float& y1) {
  const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t x =
      f2_pack(fminf(fmaxf(x0, -125.0f), 126.0f), fminf(fmaxf(x1, -125.0f), 126.0f));
  const uint64_t t = f2_add(x, magic);
  const uint64_t r = f2_sub(x, f2_sub(t, magic));
  uint64_t p = f2_fma(f2_pack(0.0551716685295105f, 0.0551716685295105f), r,
                      f2_pack(0.2426111251115799f, 0.2426111251115799f));
  p = f2_fma(p, r, f2_pack(0.6932609677314758f, 0.6932609677314758f));
  p = f2_fma(p, r, f2_pack(0.9999280571937561f, 0.9999280571937561f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Two fp32 -> packed bf16x2 (round to nearest even); lo in bits 0-15.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

}  // namespace b200
