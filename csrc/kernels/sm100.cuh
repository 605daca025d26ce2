// SPDX-License-Identifier: Apache-2.0
// Blackwell (sm_100a) primitives: mbarriers, TMA tile loads, TMEM and
// tcgen05 MMA, written as inline PTX.
//
// Rules this file enforces for the whole code base:
//   * TMA loads never use cluster multicast (kernels here also run on
//     multi-GPU communicators, and a multicast load whose tensor map reaches
//     peer memory is unsafe on this platform).  TMA stores may target peer
//     memory (plain stores).
//   * kind::f16 MMAs take A and B of the same type (both bf16).
//   * Every mbarrier wait is bounded: after ~2 s it reports failure and the
//     caller unwinds (frees TMEM, returns) instead of spinning forever.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace vccl {
namespace sm100 {

__device__ __forceinline__ uint32_t smemAddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool electOne() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .pred P;\n elect.sync _|P, 0xffffffff;\n selp.b32 %0, 1, 0, P;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void mbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemAddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fenceBarrierInit() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbarArriveExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smemAddr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbarArrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smemAddr(bar)) : "memory");
}
// try_wait without a suspend-time hint: each call returns when the phase
// completes or after the hardware's own time limit, and the callers loop
// (the bounded waits check the abort flag and the deadline between calls).
__device__ __forceinline__ bool mbarTryWait(uint64_t* bar, uint32_t phase) {
  uint32_t ok = 0;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n selp.b32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(smemAddr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t nowNs() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for `phase` to complete.  `abortFlag` (shared memory) lets one
// failed role release the others quickly.
__device__ __forceinline__ bool mbarWait(uint64_t* bar, uint32_t phase, volatile int* abortFlag,
                                         uint64_t limitNs = 2000000000ull) {
  if (mbarTryWait(bar, phase)) return true;
  const uint64_t t0 = nowNs();
  for (;;) {
    if (mbarTryWait(bar, phase)) return true;
    if (*abortFlag) return false;
    if (nowNs() - t0 > limitNs) {
      *abortFlag = 1;
      return false;
    }
  }
}

// ---- TMA (no multicast) --------------------------------------------------------
__device__ __forceinline__ void tmaPrefetchDesc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tmaLoad2d(void* smemDst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                                          int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smemAddr(smemDst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smemAddr(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// TMA store of a box from shared memory (this CTA's) to global memory, in
// the calling thread's bulk async-group.  The tensor map may describe a
// peer's memory mapped into this address space (a plain store, no multicast).
__device__ __forceinline__ void tmaStore2d(const CUtensorMap* map, const void* smemSrc, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smemAddr(smemSrc)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulkCommit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulkWaitRead0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed bulk store of this thread has completed its writes.
__device__ __forceinline__ void bulkWaitAll0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to the async proxy (TMA).
__device__ __forceinline__ void fenceProxyAsyncShared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Async-proxy global writes (TMA stores) are ordered with later generic accesses.
__device__ __forceinline__ void fenceProxyAsyncGlobal() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ---- TMEM ----------------------------------------------------------------------
// Warp-wide.  Writes the allocated TMEM address to *dstSmem.
__device__ __forceinline__ void tmemAlloc(uint32_t* dstSmem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smemAddr(dstSmem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmemRelinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmemDealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tcFenceBefore() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tcFenceAfter() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmemLoad16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmemLoad16p(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmemLoadWait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- UMMA descriptors ------------------------------------------------------------
// Shared-memory matrix descriptor for a K-major operand in the 128-byte
// swizzle layout that TMA writes (8 rows x 128 B atoms, atoms stacked every
// 1024 B).  Fields: start address >> 4 (bits 0-13), leading byte offset >> 4
// (bits 16-29, unused for this layout), stride byte offset >> 4 (bits
// 32-45), descriptor version 1 (bits 46-47), layout type 2 = 128B swizzle
// (bits 61-63).  The tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t smemDescSw128(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>(1u) << 16;             // LBO (ignored for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // SBO: 8 rows * 128 B
  d |= static_cast<uint64_t>(1u) << 46;             // version
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D fp32, A = B = bf16, both K-major.
__host__ __device__ constexpr uint32_t idescBf16F32(int m, int n) {
  return (1u << 4)                                  // D format f32
         | (1u << 7)                                // A format bf16
         | (1u << 10)                               // B format bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void mmaBf16(uint32_t tmemD, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmemD),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mmaCommit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smemAddr(bar))
               : "memory");
}

// ---- CTA pairs (clusters of two; cta_group::2) -----------------------------------
// Rank of this CTA in its cluster, the cluster's index and the number of clusters.
__device__ __forceinline__ uint32_t clusterCtaRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t clusterIdX() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t numClustersX() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address, in the cluster's shared window, of the variable at `local` in CTA `cta`.
__device__ __forceinline__ uint32_t mapaShared(const void* local, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smemAddr(local)), "r"(cta));
  return r;
}
// Arrive (release at cluster scope) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbarArriveCluster(uint32_t clusterAddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(clusterAddr) : "memory");
}
// try_wait with acquire at cluster scope: pairs with arrivals made by the
// other CTA of the cluster.
__device__ __forceinline__ bool mbarTryWaitCluster(uint64_t* bar, uint32_t phase) {
  uint32_t ok = 0;
  asm volatile(
      "{\n .reg .pred P;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P, [%1], %2;\n selp.b32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(smemAddr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded cluster-scope wait (as mbarWait).
__device__ __forceinline__ bool mbarWaitCluster(uint64_t* bar, uint32_t phase, volatile int* abortFlag,
                                                uint64_t limitNs = 2000000000ull) {
  if (mbarTryWaitCluster(bar, phase)) return true;
  const uint64_t t0 = nowNs();
  for (;;) {
    if (mbarTryWaitCluster(bar, phase)) return true;
    if (*abortFlag) return false;
    if (nowNs() - t0 > limitNs) {
      *abortFlag = 1;
      return false;
    }
  }
}
// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair's first CTA (`barCluster`: its shared::cluster
// address).  The cta_group::2 form lets a pair's loads complete on one
// barrier; no multicast.
__device__ __forceinline__ void tmaLoad2dPair(void* smemDst, const CUtensorMap* map, uint32_t barCluster, int32_t c0,
                                              int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smemAddr(smemDst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(barCluster), "r"(c0), "r"(c1)
      : "memory");
}
// Every thread of both CTAs of the cluster (all threads must call it).
__device__ __forceinline__ void clusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMEM allocation shared by the two CTAs of a pair: the same warp of both
// CTAs issues each of these.
__device__ __forceinline__ void tmemAllocPair(uint32_t* dstSmem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smemAddr(dstSmem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmemRelinquishPair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmemDeallocPair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// One MMA over the pair (issued by the pair's first CTA): A holds 128 rows in
// each CTA's shared memory and B half of the N rows in each, both at the
// descriptors' offsets; D is 128 rows x N columns in each CTA's TMEM.
__device__ __forceinline__ void mmaBf16Pair(uint32_t tmemD, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmemD),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at `bar`'s offset in every CTA of `ctaMask` once the
// pair MMAs issued so far by this thread have completed (a commit, not a load).
__device__ __forceinline__ void mmaCommitPair(uint64_t* bar, uint16_t ctaMask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smemAddr(bar)),
      "h"(ctaMask)
      : "memory");
}

}  // namespace sm100
}  // namespace vccl
