// SPDX-License-Identifier: Apache-2.0
// Row-parallel GEMM fused with reduce-scatter over NVLink.  The reference has
// no fused path; its TP test runs the row-parallel projection as a CPU GEMM
// followed by a separate all-reduce (reference:
// python/tests/test_e2e_tp.py:60-85).
//
// Every rank computes its partial product P = A * W^T.  Row r of P belongs
// to rank r / (M / n).  Instead of writing P to memory and running a
// reduce-scatter afterwards, the GEMM epilogue stores each finished tile
// directly into the owner's staging slot for this source rank (a plain
// store over NVLink for remote owners), so the transfer of early tiles
// overlaps the tensor-core work on later ones.  Two forms:
//
//  * one kernel on CTA pairs (the default where pairs cover every SM and
//    every shard is whole 256-row pair tiles): the owner's own tiles come
//    last, and their epilogue adds the peers' pushed tiles to its fp32
//    accumulator (per-half-tile arrival counters, below);
//  * push kernel + sum kernel (one-SM tiles, half pair tiles per shard,
//    VCCL_RS_TWO_KERNELS=1 or VCCL_RS_TMA=1): a short local kernel sums the
//    n slots of the rows this rank owns.
//
// The two forms share the call and free counters and may alternate from
// call to call.  For the two-kernel form, synchronisation is device-side
// and CUDA-graph safe and costs a constant
// number of system-scope operations per call: every GEMM CTA (the grid is
// always one CTA per SM) counts itself on a local counter after its
// stores, and the last one bumps done[me] on every rank once; the
// reduction waits for done[p] of this call from every source; its last
// block bumps free[me] on every rank, which the next call's GEMM waits for
// before storing into that rank's slots.
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

using dev::redAddReleaseSys;
// Two epilogue warpgroups (8 warps) share each tile: the pushes over NVLink
// are what bounds this kernel, so twice the threads keep twice the stores in
// flight.
constexpr int kRsEpiGroups = 2;
__device__ __forceinline__ void epilogueBarrier() {
  asm volatile("bar.sync 1, %0;" ::"n"(128 * kRsEpiGroups) : "memory");
}

// Optional event trace (VCCL_FUSED_TRACE=1), in the per-CTA slots the
// all-gather + GEMM trace leaves free (%globaltimer ns): 20 GEMM epilogue
// start, 21 previous call's slots freed by every rank, 22 sum over tiles of
// one epilogue warp's push time, 23 tiles pushed, 24 every tile pushed,
// 25 done signalled; reduce blocks: 26 every source's pushes arrived,
// 27 reduction written.
constexpr int kRsTraceStart = 20, kRsTraceFreed = 21, kRsTracePushNs = 22, kRsTraceTiles = 23,
              kRsTraceTilesDone = 24, kRsTraceSignalled = 25, kRsTraceArrived = 26, kRsTraceReduced = 27;
__device__ __forceinline__ void rsMark(unsigned long long* trace, int slot) {
  if (trace != nullptr) trace[blockIdx.x * dev::kFusedTraceSlots + slot] = dev::globalTimerNs();
}

// Each tile row goes to its owner's slot; rows leave the SM as contiguous
// 128-byte segments (see gemm::storeAccRows).
struct EpiPushRS {
  char* dest[dev::kMaxRanks];  // owner q's slot for this source rank
  int rowsPerRank;
  int ldn;  // N
  unsigned long long* trace;  // optional event trace (one warp's push time per tile)
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const gemm::TileInfo& ti, const gemm::GemmShape& s,
                                             int laneRow, int cBegin, uint4* st) const {
    const bool timed = trace != nullptr && laneRow == 0 && cBegin == 0;
    const unsigned long long t0 = timed ? dev::globalTimerNs() : 0ull;
    const size_t pitch = static_cast<size_t>(ldn) * 2;
    gemm::storeAccRows<SPAN>(tmemAcc, ti, s, laneRow, cBegin, st, [&](int row) {
      const int owner = row / rowsPerRank;
      return dest[owner] + static_cast<size_t>(row - owner * rowsPerRank) * pitch;
    });
    if (timed) {
      unsigned long long* t = trace + blockIdx.x * dev::kFusedTraceSlots;
      t[kRsTracePushNs] += dev::globalTimerNs() - t0;
      t[kRsTraceTiles] += 1;
    }
  }
};

// Same pushes through the TMA (VCCL_RS_TMA=1): each epilogue warp stages a
// 32-row x 64-column bf16 box in its row stage (whose XOR layout is the
// TMA's 128-byte swizzle) and one lane stores it into the owner's slot with
// cp.async.bulk.tensor, so the warp moves on while the copy engine writes
// over NVLink.  One tensor map per owner (its slot for this source rank,
// [rowsPerRank, N], box 64 x 32); plain stores, no multicast.  Needs
// 64-column passes (tile width / epilogue groups >= 64) and rowsPerRank a
// multiple of 32 (a warp's 32 rows then have one owner).
struct EpiPushRSTma {
  CUtensorMap map[dev::kMaxRanks];
  int rowsPerRank;
  unsigned long long* trace;  // optional event trace (one warp's staging time per tile)
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const gemm::TileInfo& ti, const gemm::GemmShape& s,
                                             int laneRow, int cBegin, uint4* st) const {
    // launchGemm instantiates every tile width; the host only picks this
    // epilogue for widths whose per-group span is a multiple of 64.
    if constexpr (SPAN % 64 == 0) store<SPAN>(tmemAcc, ti, s, laneRow, cBegin, st);
  }
  template <int SPAN>
  __device__ __forceinline__ void store(uint32_t tmemAcc, const gemm::TileInfo& ti, const gemm::GemmShape& s,
                                        int laneRow, int cBegin, uint4* st) const {
    const int lane = laneRow & 31;
    const int warpRow0 = ti.row0 + (laneRow & ~31);
    if (warpRow0 >= s.M) return;  // M is a multiple of 32 here: a warp's rows are all valid or all past M
    const bool timed = trace != nullptr && laneRow == 0 && cBegin == 0;
    const unsigned long long t0 = timed ? dev::globalTimerNs() : 0ull;
    const int owner = warpRow0 / rowsPerRank;
    const int slotRow = warpRow0 - owner * rowsPerRank;
#pragma unroll 1
    for (int c = cBegin; c < cBegin + SPAN && ti.col0 + c < s.N; c += 64) {  // no store starts past N
      uint32_t r[64];
#pragma unroll
      for (int i = 0; i < 4; i++) sm100::tmemLoad16p(tmemAcc + c + 16 * i, r + 16 * i);
      sm100::tmemLoadWait();
      if (lane == 0) sm100::bulkWaitRead0();  // the previous box has left the stage
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; j++) gemm::stagePut<8>(st, lane, j, gemm::packChunk(r + 8 * j));
      sm100::fenceProxyAsyncShared();
      __syncwarp();
      if (lane == 0) {
        sm100::tmaStore2d(&map[owner], st, ti.col0 + c, slotRow);
        sm100::bulkCommit();
      }
    }
    if (lane == 0) sm100::bulkWaitRead0();  // the stage is free when the tile is handed back
    __syncwarp();
    if (timed) {
      unsigned long long* t = trace + blockIdx.x * dev::kFusedTraceSlots;
      t[kRsTracePushNs] += dev::globalTimerNs() - t0;
      t[kRsTraceTiles] += 1;
    }
  }
};

template <bool kTmaStores>
struct RsHooksT : gemm::PairNoHooks {
  static constexpr int kEpiGroups = kRsEpiGroups;
  // Pair tiles walk all row tiles of a column before the next column, so a
  // wave's pushes go to every owner at once (no owner's links are a hot spot).
  __device__ __forceinline__ gemm::TileInfo pairTileAt(const gemm::GemmShape& s, int t, int, int cta) const {
    return gemm::pairTile(s, t, s.tilesM, cta);
  }
  DevComm c;
  unsigned long long* trace;  // optional event trace
  // Every rank's reduction must have consumed the previous call's pushes
  // (free[q] counts calls rank q has finished reducing).
  __device__ __forceinline__ bool beforeTiles(uint32_t*, volatile int* abortFlag) const {
    __shared__ int sFail;
    if (threadIdx.x == 64) {
      sFail = 0;
      if (trace != nullptr) {
        unsigned long long* t = trace + blockIdx.x * dev::kFusedTraceSlots;
        t[kRsTracePushNs] = 0;
        t[kRsTraceTiles] = 0;
      }
      rsMark(trace, kRsTraceStart);
      const uint32_t k = dev::ctrlAt<uint32_t>(c, c.rank, dev::kRsGemmCallsOff)[blockIdx.x];
      const uint32_t* freeCnt = dev::ctrlAt<uint32_t>(c, c.rank, dev::kRsFreeOff);
      for (int q = 0; q < c.nranks; q++)
        if (!dev::waitAcquire(c, freeCnt + q, k, dev::kWhereFused, 100 + q, 64)) sFail = 1;
      rsMark(trace, kRsTraceFreed);
    }
    epilogueBarrier();
    return sFail == 0 && !*abortFlag;
  }
  // Each CTA makes its pushes visible system-wide and counts itself locally;
  // the last CTA of the call tells every rank once (done[me] += 1).
  __device__ __forceinline__ void afterTiles(uint32_t*, volatile int*) const {
    if constexpr (kTmaStores) {
      // this warp's TMA stores have written their data, ordered before the release below
      if ((threadIdx.x & 31) == 0) {
        sm100::bulkWaitAll0();
        sm100::fenceProxyAsyncGlobal();
      }
      __syncwarp();
    }
    epilogueBarrier();
    if (threadIdx.x == 64) {
      rsMark(trace, kRsTraceTilesDone);
      uint32_t* calls = dev::ctrlAt<uint32_t>(c, c.rank, dev::kRsGemmCallsOff) + blockIdx.x;
      const uint32_t k = *calls;
      dev::fenceSys();
      const uint32_t old = atomicAdd(dev::ctrlAt<uint32_t>(c, c.rank, dev::kRsLocalDoneOff), 1u);
      if (old + 1u == (k + 1u) * gridDim.x) {
        dev::fenceSys();
        for (int q = 0; q < c.nranks; q++)
          redAddReleaseSys(dev::ctrlAt<uint32_t>(c, q, dev::kRsDoneOff) + c.rank, 1u);
      }
      *calls = k + 1u;
      rsMark(trace, kRsTraceSignalled);
    }
  }
};

using RsHooks = RsHooksT<false>;

// ---- one kernel on CTA pairs: pushes, then the reduction in the owner's epilogue ----
//
// Every rank walks its pair tiles starting at the rows of rank me + 1 and
// ending with its own rows, in shard-aligned groups.  At any moment the
// ranks push to different owners (no owner's links take every sender at
// once), and the last tiles, this rank's own rows, push nothing.  A CTA
// that pushed a 128-row half tile to owner q bumps q's arrival counter for
// that half tile (release, after all eight epilogue warps stored).  For its
// own rows the epilogue waits until the n - 1 other ranks' halves of that
// tile have arrived, adds them (bf16, from its slots) to its fp32
// accumulator and writes the output rows: no second kernel, and this rank's
// own partial is never rounded to bf16 before the sum.
//
// Per call: CTAs first wait until every owner has read the previous call's
// pushes (free[q]), as the two-kernel path does; after their tiles, the last
// CTA of this rank tells every rank once that it has read its slots.
// Arrival counters are monotonic, and calls of different shapes use
// different sets of them, so the owner keeps, per half tile, the count it has
// already consumed: a call's pushes have all landed when the counter is
// consumed + (n - 1) (senders of the next call wait for free[owner], which
// comes after the owner consumed every half of this call).  The GEMM call
// count and local done count advance as the two-kernel path expects, so the
// two paths can alternate on one communicator.

struct EpiRsPair {
  DevComm c;
  __nv_bfloat16* out;  // [rowsPerRank, N], this rank's rows of the sum
  size_t slotBytes;    // one source's slot in an owner's fused region
  int rowsPerRank;
  int ldn;             // N
  int tilesN;          // 256-wide column tiles
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const gemm::TileInfo& ti, const gemm::GemmShape& s,
                                             int laneRow, int cBegin, uint4* st) const {
    if (ti.row0 >= s.M) return;  // the second CTA's half of a pair tile past M (uniform over the warps)
    const int me = c.rank, n = c.nranks;
    const int owner = ti.row0 / rowsPerRank;
    const int half = ((ti.row0 - owner * rowsPerRank) / gemm::kBM) * tilesN + ti.tn;
    const size_t pitch = static_cast<size_t>(ldn) * 2;
    if (owner != me) {
      char* dst = c.fused[owner] + static_cast<size_t>(me) * slotBytes;
      gemm::storeAccRows<SPAN>(tmemAcc, ti, s, laneRow, cBegin, st, [&](int row) {
        return dst + static_cast<size_t>(row - owner * rowsPerRank) * pitch;
      });
      epilogueBarrier();  // every epilogue warp's stores of this half tile are issued
      if (threadIdx.x == 64) {
        dev::fenceSys();
        redAddReleaseSys(dev::ctrlAt<uint32_t>(c, owner, dev::kRsArriveOff) + half, 1u);
      }
      return;
    }
    // Own rows: wait for the other ranks' pushes of this half tile, then sum.
    const int lane = laneRow & 31;
    uint32_t* consumed = dev::ctrlAt<uint32_t>(c, me, dev::kRsConsumedOff) + half;
    const uint32_t target = *consumed + static_cast<uint32_t>(n - 1);
    if (lane == 0)
      (void)dev::waitAcquire(c, dev::ctrlAt<uint32_t>(c, me, dev::kRsArriveOff) + half, target, dev::kWhereFused,
                             600 + owner, 64);
    __syncwarp();
    constexpr int CW = SPAN < 64 ? SPAN : 64;
    constexpr int NC = CW / 8;
    const int warpRow0 = ti.row0 + (laneRow & ~31);
    const int row = warpRow0 + lane;
    const size_t rowOff = static_cast<size_t>(row - me * rowsPerRank) * pitch;
    const char* slots = c.fused[me];
    char* obase = reinterpret_cast<char*>(out);
#pragma unroll 1
    for (int cc = cBegin; cc < cBegin + SPAN; cc += CW) {
      uint32_t r[CW];
#pragma unroll
      for (int i = 0; i < CW / 16; i++) sm100::tmemLoad16p(tmemAcc + cc + 16 * i, r + 16 * i);
      sm100::tmemLoadWait();
      float acc[CW];
#pragma unroll
      for (int i = 0; i < CW; i++) acc[i] = __uint_as_float(r[i]);
      const int col0 = ti.col0 + cc;
      if (row < s.M) {
        for (int p = 0; p < n; p++) {
          if (p == me) continue;
          const char* src = slots + static_cast<size_t>(p) * slotBytes + rowOff + static_cast<size_t>(col0) * 2;
#pragma unroll
          for (int j = 0; j < NC; j++) {
            if (col0 + 8 * j >= s.N) break;
            const uint4 v = dev::ldCG(src + 16 * j);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float2 f = __bfloat1622float2(h[e]);
              acc[8 * j + 2 * e] += f.x;
              acc[8 * j + 2 * e + 1] += f.y;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < NC; j++) {
        uint4 o;
        o.x = gemm::packBf16(acc[8 * j], acc[8 * j + 1]);
        o.y = gemm::packBf16(acc[8 * j + 2], acc[8 * j + 3]);
        o.z = gemm::packBf16(acc[8 * j + 4], acc[8 * j + 5]);
        o.w = gemm::packBf16(acc[8 * j + 6], acc[8 * j + 7]);
        gemm::stagePut<NC>(st, lane, j, o);
      }
      gemm::stageFlush<NC>(st, lane, [&](int rr, int ch, uint4 v) {
        const int orow = warpRow0 + rr, col = col0 + ch * 8;
        if (orow < s.M && col < s.N)
          *reinterpret_cast<uint4*>(obase + static_cast<size_t>(orow - me * rowsPerRank) * pitch +
                                    static_cast<size_t>(col) * 2) = v;
      });
    }
    epilogueBarrier();  // every epilogue warp has read `consumed`
    if (threadIdx.x == 64) *consumed = target;
  }
};

struct RsPairHooks : gemm::PairNoHooks {
  static constexpr int kEpiGroups = kRsEpiGroups;
  DevComm c;
  int pairStartTm;    // first pair row: the rows of rank me + 1
  int pairGroupRows;  // shard-aligned tile groups
  __device__ __forceinline__ gemm::TileInfo pairTileAt(const gemm::GemmShape& s, int t, int, int cta) const {
    return gemm::pairTileFrom(s, t, pairGroupRows, pairStartTm, cta);
  }
  // Every owner must have read the previous call's pushes (free[q] counts
  // calls in which rank q finished with its slots).
  __device__ __forceinline__ bool beforeTiles(uint32_t*, volatile int* abortFlag) const {
    __shared__ int sFail;
    if (threadIdx.x == 64) {
      sFail = 0;
      const uint32_t k = dev::ctrlAt<uint32_t>(c, c.rank, dev::kRsGemmCallsOff)[blockIdx.x];
      const uint32_t* freeCnt = dev::ctrlAt<uint32_t>(c, c.rank, dev::kRsFreeOff);
      for (int q = 0; q < c.nranks; q++)
        if (!dev::waitAcquire(c, freeCnt + q, k, dev::kWhereFused, 100 + q, 64)) sFail = 1;
    }
    epilogueBarrier();
    return sFail == 0 && !*abortFlag;
  }
  // This CTA's own-row tiles have read their slots; the last CTA of the call
  // tells every rank once (free[me] += 1) and resets the CTA count.
  __device__ __forceinline__ void afterTiles(uint32_t*, volatile int*) const {
    epilogueBarrier();
    if (threadIdx.x == 64) {
      const int me = c.rank;
      uint32_t* calls = dev::ctrlAt<uint32_t>(c, me, dev::kRsGemmCallsOff) + blockIdx.x;
      atomicAdd(dev::ctrlAt<uint32_t>(c, me, dev::kRsLocalDoneOff), 1u);  // the two-kernel path's CTA count
      *calls = *calls + 1u;
      dev::fenceSys();
      uint32_t* cnt = dev::ctrlAt<uint32_t>(c, me, dev::kRsPairFreeOff);
      if (atomicAdd(cnt, 1u) == gridDim.x - 1u) {
        *cnt = 0u;  // every CTA of this call has counted (the next call starts after this kernel)
        dev::fenceSys();
        for (int q = 0; q < c.nranks; q++) redAddReleaseSys(dev::ctrlAt<uint32_t>(c, q, dev::kRsFreeOff) + me, 1u);
      }
    }
  }
};

// out[rowsPerRank, N] = sum over sources of my slots.
__global__ void __launch_bounds__(512) rsReduce(DevComm c, char* out, size_t elems, size_t slotBytes,
                                                unsigned long long* trace) {
  __shared__ uint32_t sK;
  __shared__ int sFail;
  const int n = c.nranks, me = c.rank;
  if (threadIdx.x == 0) {
    sK = dev::ctrlAt<uint32_t>(c, me, dev::kRsReduceCallsOff)[blockIdx.x];
    sFail = 0;
  }
  __syncthreads();
  const uint32_t k = sK;
  if (threadIdx.x < n) {
    const uint32_t* done = dev::ctrlAt<uint32_t>(c, me, dev::kRsDoneOff);
    if (!dev::waitAcquire(c, done + threadIdx.x, k + 1u, dev::kWhereFused, 200 + threadIdx.x, 32)) sFail = 1;
  }
  __syncthreads();
  if (sFail) return;
  if (threadIdx.x == 0) rsMark(trace, kRsTraceArrived);
  size_t lo, hi;
  dev::blockRange(elems, gridDim.x, blockIdx.x, 8, &lo, &hi);
  if (lo < hi) {
    const char* slots = c.fused[me];
    dev::reduceInto<__nv_bfloat16, dev::kSum, true>(
        n, me, out + lo * 2, nullptr, slots + me * slotBytes + lo * 2,
        [&](int p) { return slots + p * slotBytes + lo * 2; }, hi - lo, false, 1.0, false);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Slot reads are done; the last block of the call frees the slots on
    // every rank (free[me] += 1).
    __threadfence();
    const uint32_t old = atomicAdd(dev::ctrlAt<uint32_t>(c, me, dev::kRsLocalFreeOff), 1u);
    if (old + 1u == (k + 1u) * gridDim.x)
      for (int q = 0; q < n; q++) redAddReleaseSys(dev::ctrlAt<uint32_t>(c, q, dev::kRsFreeOff) + me, 1u);
    dev::ctrlAt<uint32_t>(c, me, dev::kRsReduceCallsOff)[blockIdx.x] = k + 1u;
    rsMark(trace, kRsTraceReduced);
  }
}

}  // namespace fused
}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclGemmReduceScatter(const void* A, const void* W, void* out, int M, int N, int K,
                                              vcclComm_t comm, vcclStream_t stream) {
  TraceRange trace("vccl GemmReduceScatter");
  if (comm == nullptr || A == nullptr || W == nullptr || out == nullptr || M <= 0 || N <= 0 || K <= 0)
    return vcclInvalidArgument;
  if ((N % 16) != 0 || (K % 8) != 0 || (reinterpret_cast<uintptr_t>(out) & 15u) != 0) return vcclInvalidArgument;
  if (comm->aborted.load() || !comm->dev) return vcclInvalidUsage;
  const int n = comm->nranks;
  if (M % n != 0) {
    VERR("vcclGemmReduceScatter: M (%d) must be divisible by the number of ranks (%d)", M, n);
    return vcclInvalidArgument;
  }
  vcclResult_t st = comm->pollDeviceStatus();
  if (st != vcclSuccess) {
    comm->noteError(st);
    return vcclInvalidUsage;
  }
  cudaSetDevice(comm->dev->device);
  if (!devicePointers(comm->dev->device, {A, W, out}, "vcclGemmReduceScatter")) return vcclInvalidArgument;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  OrderedLaunch ord(comm->dev.get(), s);
  const int bnEnv = static_cast<int>(gemm::envLongGemm("VCCL_GEMM_BN"));
  if (n == 1) {  // nothing to scatter: the plain GEMM (split-K, CTA pairs or one-SM tiles)
    comm->noteCall("gemm + reduce-scatter", "one rank: GEMM", static_cast<size_t>(M) * N * 2);
    return gemm::gemmWithScratch("vcclGemmReduceScatter", A, W, out, M, N, K, false, s);
  }
  const int rowsPerRank = M / n;
  if (M <= comm->dev->fusedSmallRows && (static_cast<size_t>(rowsPerRank) * N * 2) % 8 == 0) {
    // Few rows: (split-K) GEMM into local scratch, then the LL or push
    // reduce-scatter; cheaper than the persistent fused kernel at this size.
    const size_t pBytes = (static_cast<size_t>(M) * N * 2 + 255) / 256 * 256;
    const size_t wsBytes = gemm::gemmAutoScratchBytes(M, N, K, bnEnv, true);
    gemm::Scratch sc;
    if (!gemm::acquireScratch(s, pBytes + wsBytes, &sc)) {
      VERR("vcclGemmReduceScatter: cannot allocate %zu bytes of scratch", pBytes + wsBytes);
      return vcclSystemError;
    }
    char* p = static_cast<char*>(sc.p);
    cudaError_t e =
        gemm::gemmAuto(A, W, p, M, N, K, false, s, bnEnv, true, reinterpret_cast<float*>(p + pBytes), sc.sems);
    if (e == cudaSuccess) {
      dev::CollArgs a{};
      a.send = p;
      a.recv = static_cast<char*>(out);
      a.count = static_cast<size_t>(rowsPerRank) * N;
      a.root = -1;
      a.premul = 0;
      a.avg = 0;
      a.scalar = 1.0;
      e = launchReduceScatter(launchCtxFor(*comm->dev, s), vcclBfloat16, dev::kSum, a);
    }
    gemm::releaseScratch(sc);
    if (e != cudaSuccess) {
      VERR("vcclGemmReduceScatter (small): %s", cudaGetErrorString(e));
      return vcclInvalidArgument;
    }
    comm->noteCall("gemm + reduce-scatter", "small: GEMM, then reduce-scatter", static_cast<size_t>(M) * N * 2);
    return vcclSuccess;
  }
  const size_t slotBytes = (static_cast<size_t>(rowsPerRank) * N * 2 + 255) / 256 * 256;
  const dev::DevComm& dc = comm->dev->dc;
  // One kernel on CTA pairs (pushes + reduction in the owner's epilogue) when
  // the pair grid covers every SM, each pair tile's 256 rows have one owner
  // and the owner's tiles fit the arrival counters.  Whole pair tiles per
  // shard put every rank's own rows last in each pair's tile sequence, so a
  // pair only waits after all its pushes are out.  With half pair tiles
  // (rowsPerRank = 128 mod 256) own rows come mid-sequence, and a pair
  // waiting on them holds back its later pushes, which other ranks' pairs
  // may be waiting for: at 8 ranks with 56 column tiles that closes a cycle
  // (a model of the tile walk shows it); those shapes take the two-kernel
  // path, whose pushes never wait.
  if (slotBytes * n <= dc.fusedBytes / 2 && rowsPerRank % gemm::kPairBM == 0 &&
      gemm::envLongGemm("VCCL_RS_TMA") == 0 && gemm::envLongGemm("VCCL_RS_TWO_KERNELS") == 0) {
    const int pairs = gemm::pairClustersFor<fused::EpiRsPair, fused::RsPairHooks>();
    const int tilesN = (N + gemm::kPairBN - 1) / gemm::kPairBN;
    if (2 * pairs == gemm::smCount() && pairs <= dev::kMaxFusedCtas / 2 &&
        (rowsPerRank / gemm::kBM) * tilesN <= dev::kRsMaxHalves && gemm::pairPreferred(M, N, bnEnv, pairs)) {
      fused::EpiRsPair epi;
      epi.c = dc;
      epi.out = static_cast<__nv_bfloat16*>(out);
      epi.slotBytes = slotBytes;
      epi.rowsPerRank = rowsPerRank;
      epi.ldn = N;
      epi.tilesN = tilesN;
      fused::RsPairHooks hooks;
      hooks.c = dc;
      const int tilesM = (M + gemm::kPairBM - 1) / gemm::kPairBM;
      hooks.pairStartTm = (((comm->rank + 1) % n) * rowsPerRank / gemm::kPairBM) % tilesM;
      const int shardPairTiles = rowsPerRank / gemm::kPairBM;
      hooks.pairGroupRows = 1;
      for (int gsz = 16; gsz >= 1; gsz /= 2)
        if (shardPairTiles % gsz == 0) {
          hooks.pairGroupRows = gsz;
          break;
        }
      cudaError_t e = gemm::launchGemmPair(A, W, M, N, K, epi, s, nullptr, hooks, pairs);
      if (e != cudaSuccess) {
        VERR("vcclGemmReduceScatter (pairs) launch: %s", cudaGetErrorString(e));
        return gemm::launchResult(e);
      }
      comm->noteCall("gemm + reduce-scatter", "one kernel on CTA pairs", static_cast<size_t>(M) * N * 2);
      return vcclSuccess;
    }
  }
  if (slotBytes * n > dc.fusedBytes / 2) {
    VERR("vcclGemmReduceScatter: %zu staging bytes exceed VCCL_FUSED_BUFFSIZE/2", slotBytes * n);
    return vcclInvalidArgument;
  }
  cudaError_t e = cudaSuccess;
  bool tma = gemm::envLongGemm("VCCL_RS_TMA") != 0 && rowsPerRank % 32 == 0;
  // CTA pairs (256 x 256 tiles) where they take no more waves than one-SM
  // tiles; the grid is fixed either way (the done counters count CTAs).
  const int pairs = tma ? gemm::pairClustersFor<fused::EpiPushRSTma, fused::RsHooksT<true>>()
                        : gemm::pairClustersFor<fused::EpiPushRS, fused::RsHooks>();
  // The per-CTA call counters need the same grid on every call: pairs only
  // when they cover every SM, as the one-SM grid does.
  const bool usePair = 2 * pairs == gemm::smCount() && gemm::pairPreferred(M, N, bnEnv, pairs);
  const int ctas = usePair ? 2 * pairs : gemm::smCount();
  if (ctas > dev::kMaxFusedCtas) return vcclInternalError;
  const int bn = usePair ? gemm::kPairBN : bnEnv > 0 ? bnEnv : gemm::pickBN(M, N);
  if (tma && !usePair && bn / fused::kRsEpiGroups < 64) tma = false;
  if (tma) {
    fused::EpiPushRSTma epi{};
    epi.rowsPerRank = rowsPerRank;
    epi.trace = comm->dev->fusedTrace;
    for (int q = 0; q < n && tma; q++)
      tma = gemm::makeMapKMajor(&epi.map[q], dc.fused[q] + comm->rank * slotBytes, rowsPerRank, N, 32);
    if (tma) {
      fused::RsHooksT<true> hooks;
      hooks.c = dc;
      hooks.trace = comm->dev->fusedTrace;
      e = usePair ? gemm::launchGemmPair(A, W, M, N, K, epi, s, nullptr, hooks, pairs)
                  : gemm::launchGemm(A, W, M, N, K, epi, hooks, s, bn, -ctas);
    }
  }
  if (!tma) {
    fused::EpiPushRS epi;
    for (int q = 0; q < dev::kMaxRanks; q++) epi.dest[q] = q < n ? dc.fused[q] + comm->rank * slotBytes : nullptr;
    epi.rowsPerRank = rowsPerRank;
    epi.ldn = N;
    epi.trace = comm->dev->fusedTrace;
    fused::RsHooks hooks;
    hooks.c = dc;
    hooks.trace = comm->dev->fusedTrace;
    e = usePair ? gemm::launchGemmPair(A, W, M, N, K, epi, s, nullptr, hooks, pairs)
                : gemm::launchGemm(A, W, M, N, K, epi, hooks, s, bnEnv, -ctas);
  }
  if (e != cudaSuccess) {
    VERR("vcclGemmReduceScatter GEMM launch: %s", cudaGetErrorString(e));
    return gemm::launchResult(e);
  }
  fused::rsReduce<<<dev::kFusedReduceBlocks, 512, 0, s>>>(
      dc, static_cast<char*>(out), static_cast<size_t>(rowsPerRank) * N, slotBytes, comm->dev->fusedTrace);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    VERR("vcclGemmReduceScatter reduce launch: %s", cudaGetErrorString(e));
    return vcclUnhandledError;
  }
  comm->noteCall("gemm + reduce-scatter", tma ? "push (TMA stores) + sum kernel" : "push + sum kernel",
                 static_cast<size_t>(M) * N * 2);
  return vcclSuccess;
}
