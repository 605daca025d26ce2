// SPDX-License-Identifier: Apache-2.0
// All-gather fused into a column-parallel GEMM.  The reference's TP test
// gathers with a separate all_gather before the CPU GEMM (reference:
// python/tests/test_e2e_tp.py:60-85, python/vccl/torch_comm.py:141-158).
//
// Each rank holds X_shard[M/n, K] (sequence-parallel activations) and needs
// out = AllGather(X)[M, K] * W^T.  One persistent kernel does both: two
// extra warps per CTA first stage this rank's shard into its symmetric
// full-X buffer, then pull every peer's shard over NVLink into the same
// buffer, bumping a per-shard arrival counter; the TMA producer gates each A
// tile on the counters of the shards it covers.  Tiles are visited starting
// at the local shard, so the tensor cores start before any remote byte has
// arrived and later shards arrive while earlier ones are multiplied.
//
// Remote data is read with plain per-thread loads from peer memory into
// this GPU's memory; the TMA only ever reads local memory (and never uses
// multicast).
#include <cuda_runtime.h>

#include "common/log.h"
#include "common/trace.h"
#include "fused/gemm_launch.cuh"
#include "kernels/collectives.cuh"
#include "runtime/comm.h"
#include "runtime/launch.h"
#include "vccl_tp.h"

namespace vccl {
namespace fused {

using dev::DevComm;

__device__ __forceinline__ void redAddRelease(uint32_t* p, uint32_t v, bool sys) {
  if (sys)
    dev::redAddReleaseSys(p, v);
  else
    dev::redAddReleaseGpu(p, v);
}
__device__ __forceinline__ void fenceProxyAsync() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void copyWarpsBarrier() { asm volatile("bar.sync 2, 64;" ::: "memory"); }

// Copy by the 64 copy-warp threads, 16 x 16 B in flight per thread: the
// staging of the own shard and the pulls of the peers' shards are
// latency-bound (a 4-GPU trace had the own 16 MiB shard staged only after
// ~20 us with 8 in flight).
__device__ __forceinline__ void groupCopy(char* dst, const char* src, size_t bytes, int tid) {
  constexpr int U = 16;
  const size_t n16 = bytes / 16;
  size_t i = tid;
  for (; i + (U - 1) * 64 < n16; i += U * 64) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) v[u] = dev::ldCG(src + (i + u * 64) * 16);
#pragma unroll
    for (int u = 0; u < U; u++) dev::stG(dst + (i + u * 64) * 16, v[u]);
  }
  for (; i < n16; i += 64) dev::stG(dst + i * 16, dev::ldCG(src + i * 16));
}

struct AgHooks : gemm::PairNoHooks {
  static constexpr int kExtraWarps = 2;
  DevComm c;
  const char* xShard;  // this rank's input rows [shardRows, K]
  size_t xOff;         // offset of the full-X buffer in the fused region
  int shardRows;
  int K;
  int startTm;         // first tile row of this rank's shard
  int groupRows;       // row tiles per tile group (divides the shard's tiles when possible)
  int pairStartTm;     // the same two in 256-row pair tiles (CTA-pair kernel)
  int pairGroupRows;
  // CTA-pair kernel only: this rank's shard read in place through its own
  // tensor map, so the own tiles start without waiting for the staging copy
  // (which the peers still pull from).  ownDirect = 0 disables it.
  CUtensorMap ownMap;
  int ownDirect;
  uint32_t ctas;       // fixed grid size
  // Optional event trace (VCCL_FUSED_TRACE=1), kFusedTraceSlots times per CTA
  // from %globaltimer: 0 kernel start, 1 previous call's shard taken by every
  // peer, 2 own slice staged, 3..9 pull of the s-th peer shard done,
  // 10..17 first tile of the s-th shard (own shard s = 0) released to the
  // TMA producer, 18 kernel end.
  unsigned long long* trace;

  __device__ __forceinline__ void mark(int slot) const {
    if (trace != nullptr) trace[blockIdx.x * dev::kFusedTraceSlots + slot] = dev::globalTimerNs();
  }

  __device__ __forceinline__ uint32_t* ctrl(int rank, size_t off) const {
    return dev::ctrlAt<uint32_t>(c, rank, off);
  }
  __device__ __forceinline__ void setup(uint32_t* hs) const {
    hs[0] = ctrl(c.rank, dev::kAgCallsOff)[blockIdx.x];
    mark(0);
  }
  __device__ __forceinline__ void teardown(uint32_t* hs) const {
    ctrl(c.rank, dev::kAgCallsOff)[blockIdx.x] = hs[0] + 1u;
    mark(18);
  }
  // Row tiles start at this rank's shard and wrap around, in groups that
  // share weight tiles (see gemm::groupedTile).
  __device__ __forceinline__ gemm::TileInfo tileAt(const gemm::GemmShape& s, int t, int BN) const {
    return gemm::groupedTile(s, t, BN, groupRows, startTm);
  }
  __device__ __forceinline__ gemm::TileInfo pairTileAt(const gemm::GemmShape& s, int t, int, int cta) const {
    return gemm::pairTileFrom(s, t, pairGroupRows, pairStartTm, cta);
  }
  // Own-shard rows of a CTA whose 128 rows lie inside this rank's shard.
  __device__ __forceinline__ bool ownRows(const gemm::TileInfo& ti, const gemm::GemmShape&) const {
    return ownDirect != 0 && ti.row0 / shardRows == c.rank;
  }
  __device__ __forceinline__ const CUtensorMap* aMapFor(const gemm::TileInfo& ti, const CUtensorMap* mapA,
                                                        int* row) const {
    // ownDirect needs shardRows % 256 == 0, so a pair tile's rows lie in one shard
    if (ownDirect != 0 && ti.row0 / shardRows == c.rank) {
      *row = ti.row0 - c.rank * shardRows;
      return &ownMap;
    }
    return mapA;
  }
  __device__ __forceinline__ bool beforeLoad(const gemm::TileInfo& ti, const gemm::GemmShape& s, uint32_t* hs,
                                             volatile int*) const {
    if (ownRows(ti, s)) return true;  // read in place: nothing to wait for
    const uint32_t k = hs[0];
    const int last = (ti.row0 + gemm::kBM < s.M ? ti.row0 + gemm::kBM : s.M) - 1;
    for (int q = ti.row0 / shardRows; q <= last / shardRows; q++) {
      // Own shard: staged by every CTA (ready[me] bumps once per call);
      // remote shard q: every CTA pulled its slice (local counter).
      const bool own = q == c.rank;
      const uint32_t* flag = own ? ctrl(c.rank, dev::kAgReadyOff) + q : ctrl(c.rank, dev::kAgLocalReadyOff) + q;
      if (!dev::waitAcquire(c, flag, own ? k + 1u : (k + 1u) * ctas, dev::kWhereFused, 300 + q, 64)) return false;
      if (trace != nullptr) {
        unsigned long long* t = trace + blockIdx.x * dev::kFusedTraceSlots;
        const int slot = 10 + (q - c.rank + c.nranks) % c.nranks;
        if (t[slot] < t[0]) t[slot] = dev::globalTimerNs();  // first release of this shard in this call
      }
    }
    fenceProxyAsync();
    return true;
  }
  __device__ __forceinline__ void extraRole(uint32_t* hs, volatile int* abortFlag) const {
    const int tid = threadIdx.x - gemm::baseThreads<AgHooks>();  // 0..63
    const int n = c.nranks, me = c.rank;
    const uint32_t k = hs[0];
    const size_t rowBytes = static_cast<size_t>(K) * 2;
    char* xfull = c.fused[me] + xOff;
    __shared__ int sFail;
    // Rows of each shard this CTA moves.
    const int per = (shardRows + static_cast<int>(ctas) - 1) / static_cast<int>(ctas);
    const int r0 = blockIdx.x * per < shardRows ? blockIdx.x * per : shardRows;
    const int r1 = r0 + per < shardRows ? r0 + per : shardRows;
    // 1. every peer must have finished pulling the previous call's shard
    //    (taken[p] counts calls in which rank p pulled all of my shard)
    if (tid == 0) {
      sFail = 0;
      for (int p = 0; p < n; p++)
        if (p != me && !dev::waitAcquire(c, ctrl(me, dev::kAgTakenOff) + p, k, dev::kWhereFused, 400 + p, 64))
          sFail = 1;
    }
    copyWarpsBarrier();
    if (sFail) {
      *abortFlag = 1;
      return;
    }
    if (tid == 0) mark(1);
    // 2. stage my slice of my shard; the last CTA to finish announces the
    //    shard to every rank once (me included)
    if (r1 > r0)
      groupCopy(xfull + (static_cast<size_t>(me) * shardRows + r0) * rowBytes, xShard + r0 * rowBytes,
                (r1 - r0) * rowBytes, tid);
    copyWarpsBarrier();
    if (tid == 0) {
      fenceProxyAsync();
      dev::fenceSys();
      const uint32_t old = atomicAdd(ctrl(me, dev::kAgStagedOff), 1u);
      if (old + 1u == (k + 1u) * ctas)
        for (int p = 0; p < n; p++) redAddRelease(ctrl(p, dev::kAgReadyOff) + me, 1u, true);
      mark(2);
    }
    // 3. pull my slice of every peer's shard; the last CTA to finish a shard
    //    tells its owner it may be overwritten
    for (int s = 1; s < n; s++) {
      const int q = (me + s) % n;
      if (tid == 0 && !dev::waitAcquire(c, ctrl(me, dev::kAgReadyOff) + q, k + 1u, dev::kWhereFused, 500 + q, 64))
        sFail = 1;
      copyWarpsBarrier();
      if (sFail || *abortFlag) {
        *abortFlag = 1;
        return;
      }
      const size_t off = (static_cast<size_t>(q) * shardRows + r0) * rowBytes;
      if (r1 > r0) groupCopy(xfull + off, c.fused[q] + xOff + off, (r1 - r0) * rowBytes, tid);
      copyWarpsBarrier();
      if (tid == 0) {
        fenceProxyAsync();
        __threadfence();
        const uint32_t old = atomicAdd(ctrl(me, dev::kAgLocalReadyOff) + q, 1u);
        if (old + 1u == (k + 1u) * ctas) redAddRelease(ctrl(q, dev::kAgTakenOff) + me, 1u, true);
        mark(2 + s);
      }
    }
  }
};

}  // namespace fused
}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclAllGatherGemm(const void* xShard, const void* W, void* out, int M, int N, int K,
                                          int siluMul, vcclComm_t comm, vcclStream_t stream) {
  TraceRange trace("vccl AllGatherGemm");
  if (comm == nullptr || xShard == nullptr || W == nullptr || out == nullptr || M <= 0 || N <= 0 || K <= 0)
    return vcclInvalidArgument;
  if ((N % 32) != 0 || (K % 8) != 0 ||
      ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(xShard)) & 15u) != 0)
    return vcclInvalidArgument;
  if (comm->aborted.load() || !comm->dev) return vcclInvalidUsage;
  const int n = comm->nranks;
  if (M % n != 0) {
    VERR("vcclAllGatherGemm: M (%d) must be divisible by the number of ranks (%d)", M, n);
    return vcclInvalidArgument;
  }
  vcclResult_t st = comm->pollDeviceStatus();
  if (st != vcclSuccess) {
    comm->noteError(st);
    return vcclInvalidUsage;
  }
  cudaSetDevice(comm->dev->device);
  if (!devicePointers(comm->dev->device, {xShard, W, out}, "vcclAllGatherGemm")) return vcclInvalidArgument;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  OrderedLaunch ord(comm->dev.get(), s);
  const int bnEnv = static_cast<int>(gemm::envLongGemm("VCCL_GEMM_BN"));
  cudaError_t e;
  if (n == 1) {  // the gather is the shard itself: the plain GEMM (split-K, CTA pairs or one-SM tiles)
    comm->noteCall("all-gather + gemm", "one rank: GEMM", static_cast<size_t>(M) * K * 2);
    return gemm::gemmWithScratch("vcclAllGatherGemm", xShard, W, out, M, N, K, siluMul, s);
  }
  if (M <= comm->dev->fusedSmallRows) {
    // Few rows (decode, short prefills): the gather is a few hundred KB, so
    // an LL all-gather into local scratch followed by a (split-K) GEMM beats
    // the persistent fused kernel, whose per-call synchronisation and
    // mostly idle tiles dominate at this size.
    const size_t xBytes = (static_cast<size_t>(M) * K * 2 + 255) / 256 * 256;
    const size_t wsBytes = gemm::gemmAutoScratchBytes(M, N, K, bnEnv, true);
    gemm::Scratch sc;
    if (!gemm::acquireScratch(s, xBytes + wsBytes, &sc)) {
      VERR("vcclAllGatherGemm: cannot allocate %zu bytes of scratch", xBytes + wsBytes);
      return vcclSystemError;
    }
    char* xfull = static_cast<char*>(sc.p);
    e = launchAllGather(launchCtxFor(*comm->dev, s), xShard, xfull, static_cast<size_t>(M / n) * K * 2);
    if (e == cudaSuccess)
      e = gemm::gemmAuto(xfull, W, out, M, N, K, siluMul != 0, s, bnEnv, true,
                         reinterpret_cast<float*>(xfull + xBytes), sc.sems);
    gemm::releaseScratch(sc);
    if (e != cudaSuccess) {
      VERR("vcclAllGatherGemm (small): %s", cudaGetErrorString(e));
      return vcclInvalidArgument;
    }
    comm->noteCall("all-gather + gemm", "small: LL all-gather, then GEMM", static_cast<size_t>(M) * K * 2);
    return vcclSuccess;
  }
  const dev::DevComm& dc = comm->dev->dc;
  const size_t xOff = dc.fusedBytes / 2;
  if (static_cast<size_t>(M) * K * 2 > dc.fusedBytes - xOff) {
    VERR("vcclAllGatherGemm: gathered input (%zu bytes) exceeds VCCL_FUSED_BUFFSIZE/2",
         static_cast<size_t>(M) * K * 2);
    return vcclInvalidArgument;
  }
  // CTA pairs (256 x 256 tiles) where they take no more waves than one-SM
  // tiles; either way the grid is fixed and every CTA is resident.
  const int pairs = siluMul ? gemm::pairClustersFor<gemm::EpiSiluMul, fused::AgHooks>()
                            : gemm::pairClustersFor<gemm::EpiStore, fused::AgHooks>();
  // The per-CTA call counters need the same grid on every call: pairs only
  // when they cover every SM, as the one-SM grid does.
  const bool usePair = 2 * pairs == gemm::smCount() && gemm::pairPreferred(M, N, bnEnv, pairs);
  const int ctas = usePair ? 2 * pairs : gemm::smCount();
  fused::AgHooks hooks;
  hooks.c = dc;
  hooks.xShard = static_cast<const char*>(xShard);
  hooks.xOff = xOff;
  hooks.shardRows = M / n;
  hooks.K = K;
  hooks.startTm = (comm->rank * (M / n)) / gemm::kBM;
  // Shard-aligned groups of up to 16 row tiles (the rotation by startTm then
  // keeps groups inside shards); ragged shards fall back to one row per group.
  const int shardTiles = (M / n) % gemm::kBM == 0 ? (M / n) / gemm::kBM : 0;
  int groupRows = 1;
  for (int gsz = 16; gsz >= 1; gsz /= 2)
    if (shardTiles > 0 && shardTiles % gsz == 0) {
      groupRows = gsz;
      break;
    }
  hooks.groupRows = groupRows;
  hooks.pairStartTm = (comm->rank * (M / n)) / gemm::kPairBM;
  const int shardPairTiles = (M / n) % gemm::kPairBM == 0 ? (M / n) / gemm::kPairBM : 0;
  hooks.pairGroupRows = 1;
  for (int gsz = 16; gsz >= 1; gsz /= 2)
    if (shardPairTiles > 0 && shardPairTiles % gsz == 0) {
      hooks.pairGroupRows = gsz;
      break;
    }
  hooks.ctas = static_cast<uint32_t>(ctas);
  // The own shard is read in place when it is whole pair tiles, so the two
  // CTAs of a pair always read their rows the same way; a shard of half pair
  // tiles (M / n = 128 mod 256, e.g. 1024 rows over 8 ranks) reads its staged
  // copy like the peers' shards.
  hooks.ownDirect = 0;
  if (usePair && gemm::envLongGemm("VCCL_AG_OWN_STAGED") == 0 && (M / n) % gemm::kPairBM == 0)
    hooks.ownDirect = gemm::makeMapKMajor(&hooks.ownMap, xShard, M / n, K, gemm::kBM) ? 1 : 0;
  hooks.trace = comm->dev->fusedTrace;
  const char* xfull = dc.fused[comm->rank] + xOff;
  if (siluMul) {
    gemm::EpiSiluMul epi{static_cast<__nv_bfloat16*>(out), N / 2};
    e = usePair ? gemm::launchGemmPair(xfull, W, M, N, K, epi, s, nullptr, hooks, pairs)
                : gemm::launchGemm(xfull, W, M, N, K, epi, hooks, s, bnEnv, -ctas);
  } else {
    gemm::EpiStore epi{static_cast<__nv_bfloat16*>(out), N};
    e = usePair ? gemm::launchGemmPair(xfull, W, M, N, K, epi, s, nullptr, hooks, pairs)
                : gemm::launchGemm(xfull, W, M, N, K, epi, hooks, s, bnEnv, -ctas);
  }
  if (e != cudaSuccess) {
    VERR("vcclAllGatherGemm launch: %s", cudaGetErrorString(e));
    return gemm::launchResult(e);
  }
  comm->noteCall("all-gather + gemm", usePair ? (hooks.ownDirect ? "one kernel on CTA pairs, own shard in place"
                                                                  : "one kernel on CTA pairs")
                                              : "one kernel, one-SM tiles",
                 static_cast<size_t>(M) * K * 2);
  return vcclSuccess;
}
