// SPDX-License-Identifier: Apache-2.0
// bf16 GEMM on CTA pairs: 256 x 256 output tiles computed by two SMs with
// tcgen05.mma.cta_group::2 (sm_100a).
//
//   C[M, N] = A[M, K] * B[N, K]^T      (A, B K-major; fp32 accumulation)
//
// A cluster of two CTAs owns one 256 x 256 tile at a time.  CTA c of the pair
// loads rows [128 c, 128 c + 128) of the tile's A block and rows
// [128 c, 128 c + 128) of its B block (half of the 256 output columns), so
// each SM moves 32 KB per 64-wide k-block for 4.2 MFLOP, two thirds of what a
// 128 x 256 tile on one SM moves for the same work.  The pair's first CTA
// issues every MMA (M = 256, N = 256, K = 16); the tensor cores read A and B
// from both CTAs' shared memory and leave 128 rows x 256 fp32 columns in each
// CTA's TMEM (two such accumulators alternate, all 512 columns).
//
// Warp roles, both CTAs (192 threads, more with a policy's epilogue groups
// and extra warps):
//   warp 0     TMA producer: this CTA's A and B halves into a STAGES-deep
//              ring.  Both CTAs' loads complete on the FIRST CTA's `full`
//              barrier (the cta_group::2 load form; no multicast), whose
//              producer expects the bytes of both.  Each CTA refills a slot
//              once its own `empty` barrier says the MMAs have read it.
//   warp 1     first CTA: MMA issuer.  Commits release the ring slot and
//              publish the accumulator in BOTH CTAs (commit multicast).
//              Second CTA: idle (it takes part in the TMEM allocation).
//   warps 2-5  epilogue (as the one-SM kernel), on this CTA's 128 rows; the
//              accumulator is handed back to the first CTA's `accEmpty`
//              (4 more warps per extra epilogue group, each group taking a
//              share of the 256 columns).
//   then       the policy's extra warps (the all-gather copy warps).
// The policy (PairNoHooks or a fused kernel's) supplies the tile order, may
// gate each CTA's loads on data arrival, and runs code around the tiles, as
// it does for the one-SM kernel.
// Every wait is bounded; a CTA that gives up unwinds, and both CTAs meet at a
// cluster barrier before TMEM is freed, so the MMAs writing the second CTA's
// TMEM have drained first.
#pragma once

#include "kernels/gemm_sm100.cuh"

namespace vccl {
namespace gemm {

constexpr int kPairBM = 256;  // rows of a pair tile
constexpr int kPairBN = 256;  // columns of a pair tile (each CTA loads half of B)

// Pair tile t in grouped order: groups of `groupRows` pair-row tiles, inside a
// group consecutive tiles walk the rows first and share a column tile; pair
// rows start at `startTm` and wrap around.  Row 0 of CTA `cta` is the tile's
// row 0 + 128 cta.
// With split-K (s.splits > 1), work unit t covers pair tile t % (tilesM x
// tilesN) over the k-blocks of split t / (tilesM x tilesN).
__host__ __device__ inline TileInfo pairTileFrom(const GemmShape& s, int t, int groupRows, int startTm, int cta) {
  TileInfo ti;
  const int mn = s.tilesM * s.tilesN;
  const int ks = t / mn;
  t -= ks * mn;
  const int groupTiles = groupRows * s.tilesN;
  const int g = t / groupTiles;
  const int rowsHere = s.tilesM - g * groupRows < groupRows ? s.tilesM - g * groupRows : groupRows;
  const int local = t - g * groupTiles;
  ti.tn = local / rowsHere;
  ti.tm = (g * groupRows + local % rowsHere + startTm) % s.tilesM;
  ti.row0 = ti.tm * kPairBM + kBM * cta;
  ti.col0 = ti.tn * kPairBN;
  const int nk = s.numK();
  ti.ks = ks;
  ti.kb0 = ks * nk / s.splits;
  ti.kb1 = (ks + 1) * nk / s.splits;
  return ti;
}
__host__ __device__ inline TileInfo pairTile(const GemmShape& s, int t, int groupRows, int cta) {
  return pairTileFrom(s, t, groupRows, 0, cta);
}

// The policy of the pair kernel: NoHooks' roles (gemm_sm100.cuh) plus the
// order of the pair tiles.  Policies of the fused kernels derive from it.
struct PairNoHooks : NoHooks {
  __device__ __forceinline__ TileInfo pairTileAt(const GemmShape& s, int t, int groupRows, int cta) const {
    return pairTile(s, t, groupRows, cta);
  }
  // Tensor map (and its row coordinate) this CTA reads its A rows of tile
  // `ti` through: by default the kernel's A map at the tile's rows.
  __device__ __forceinline__ const CUtensorMap* aMapFor(const TileInfo&, const CUtensorMap* mapA, int*) const {
    return mapA;
  }
};

template <int STAGES, int EPI_WARPS = 4>
using PairSmem = Smem<kPairBN / 2, STAGES, EPI_WARPS>;  // A 128 x 64 + B half 128 x 64 per stage

template <int STAGES, typename Epi, typename Hooks = PairNoHooks>
__global__ void __launch_bounds__(ctaThreads<Hooks>(), 1)
    gemmPairKernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, GemmShape s,
                   const __grid_constant__ Epi epi, const __grid_constant__ Hooks hooks, int groupRows,
                   int* errorFlag) {
  constexpr int kEpiWarps = 4 * Hooks::kEpiGroups;
  constexpr int kSpan = kPairBN / Hooks::kEpiGroups;
  using L = PairSmem<STAGES, kEpiWarps>;
  constexpr uint32_t kTmemCols = 2 * kPairBN;
  extern __shared__ __align__(1024) uint8_t smemRaw[];
  // The same offset in both CTAs: the MMA reads both CTAs' stages at the
  // descriptor's address, and the commits arrive at the barrier's offset.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smemRaw) + 1023) & ~uintptr_t(1023));
  uint64_t* fullBar = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* emptyBar = fullBar + STAGES;
  uint64_t* accFull = emptyBar + STAGES;
  uint64_t* accEmpty = accFull + 2;
  uint64_t* drainBar = accEmpty + 2;
  uint32_t* tmemSlot = reinterpret_cast<uint32_t*>(drainBar + 1);
  volatile int* abortFlag = reinterpret_cast<volatile int*>(tmemSlot + 1);
  uint32_t* hs = tmemSlot + 2;  // 8 words of policy scratch

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t cta = sm100::clusterCtaRank();  // 0: issues the MMAs
  const bool first = cta == 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; i++) {
      sm100::mbarInit(&fullBar[i], 1);  // the first CTA's producer (the second CTA's is unused)
      sm100::mbarInit(&emptyBar[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      sm100::mbarInit(&accFull[i], 1);
      sm100::mbarInit(&accEmpty[i], 2 * kEpiWarps);
    }
    sm100::mbarInit(drainBar, 1);
    *abortFlag = 0;
    hooks.setup(hs);
    sm100::fenceBarrierInit();
  }
  if (warp == 1) {
    sm100::tmemAllocPair(tmemSlot, kTmemCols);
    sm100::tmemRelinquishPair();
  }
  sm100::tcFenceBefore();
  // Both CTAs' barriers are initialised before either CTA signals the other.
  sm100::clusterSync();
  sm100::tcFenceAfter();
  const uint32_t tmemBase = *tmemSlot;
  const int numTiles = s.tilesM * s.tilesN * s.splits;
  const int pair0 = static_cast<int>(sm100::clusterIdX());
  const int pairs = static_cast<int>(sm100::numClustersX());

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (sm100::electOne()) {
      sm100::tmaPrefetchDesc(&mapA);
      sm100::tmaPrefetchDesc(&mapB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair0; t < numTiles && ok; t += pairs) {
        const TileInfo ti = hooks.pairTileAt(s, t, groupRows, static_cast<int>(cta));
        // The policy may hold this CTA's rows back until their data is there.
        if (!hooks.beforeLoad(ti, s, hs, abortFlag)) {
          *abortFlag = 1;
          ok = false;
          break;
        }
        const int bRow0 = ti.tn * kPairBN + (kPairBN / 2) * static_cast<int>(cta);
        // The policy may read this CTA's A rows through another tensor map.
        int aRow = ti.row0;
        const CUtensorMap* aMap = hooks.aMapFor(ti, &mapA, &aRow);
        for (int kb = ti.kb0; kb < ti.kb1; kb++) {
          if (!sm100::mbarWait(&emptyBar[stage], phase ^ 1u, abortFlag)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + stage * L::kStageBytes;
          uint8_t* b = a + L::kABytes;
          if (first)
            sm100::mbarArriveExpectTx(&fullBar[stage], static_cast<uint32_t>(2 * (L::kABytes + L::kBBytes)));
          const uint32_t bar = sm100::mapaShared(&fullBar[stage], 0);
          sm100::tmaLoad2dPair(a, aMap, bar, kb * kBK, aRow);
          sm100::tmaLoad2dPair(b, &mapB, bar, kb * kBK, bRow0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // After an abort, copies still in flight land before the final
      // cluster barrier: every slot is waited on through its `empty`
      // barrier only while the MMAs run, so drain through the first CTA's
      // `full` barriers with a short bound (the peer's bytes may be owed).
      if (!ok && first) {
        volatile int never = 0;
        for (int i = 0; i < STAGES; i++) sm100::mbarWait(&fullBar[i], 0, &never, 20000000ull);
      }
    }
  } else if (warp == 1) {
    if (first) {
      // ---------------- MMA issuer (first CTA) ----------------
      if (sm100::electOne()) {
        constexpr uint32_t idesc = sm100::idescBf16F32(kPairBM, kPairBN);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t accPhase = 0;
        bool ok = true;
        bool anyIssued = false;
        for (int t = pair0; t < numTiles && ok; t += pairs) {
          if (!sm100::mbarWaitCluster(&accEmpty[acc], accPhase ^ 1u, abortFlag)) {
            ok = false;
            break;
          }
          sm100::tcFenceAfter();
          const uint32_t tmemAcc = tmemBase + acc * kPairBN;
          const TileInfo ti = hooks.pairTileAt(s, t, groupRows, 0);
          for (int kb = ti.kb0; kb < ti.kb1; kb++) {
            if (!sm100::mbarWaitCluster(&fullBar[stage], phase, abortFlag)) {
              ok = false;
              break;
            }
            sm100::tcFenceAfter();
            const uint32_t aAddr = sm100::smemAddr(smem + stage * L::kStageBytes);
            const uint32_t bAddr = aAddr + L::kABytes;
            const uint64_t ad = sm100::smemDescSw128(aAddr);
            const uint64_t bd = sm100::smemDescSw128(bAddr);
#pragma unroll
            for (int k = 0; k < kBK / 16; k++)
              sm100::mmaBf16Pair(tmemAcc, ad + 2 * k, bd + 2 * k, idesc, (kb != ti.kb0 || k != 0) ? 1u : 0u);
            anyIssued = true;
            sm100::mmaCommitPair(&emptyBar[stage], 0x3);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          sm100::mmaCommitPair(&accFull[acc], 0x3);
          if (++acc == 2) {
            acc = 0;
            accPhase ^= 1u;
          }
        }
        if (!ok && anyIssued) {
          // Drain every MMA in flight (they write both CTAs' TMEM).
          sm100::mmaCommitPair(drainBar, 0x1);
          volatile int never = 0;
          sm100::mbarWait(drainBar, 0, &never, 200000000ull);
        }
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ---------------- epilogue (warps 2 .. 1 + kEpiWarps, both CTAs) ----------------
    const int quarter = warp & 3;
    const int laneRow = quarter * 32 + lane;
    const int cBegin = ((warp - 2) / 4) * kSpan;
    uint4* rowStage = reinterpret_cast<uint4*>(smem + L::kRowStageOff + (warp - 2) * kWarpStageBytes);
    const uint32_t accEmptyFirst0 = sm100::mapaShared(&accEmpty[0], 0);
    const uint32_t accEmptyFirst1 = sm100::mapaShared(&accEmpty[1], 0);
    int acc = 0;
    uint32_t accPhase = 0;
    bool ok = hooks.beforeTiles(hs, abortFlag);
    if (!ok) *abortFlag = 1;
    for (int t = pair0; t < numTiles && ok; t += pairs) {
      if (!sm100::mbarWait(&accFull[acc], accPhase, abortFlag)) {
        ok = false;
        break;
      }
      sm100::tcFenceAfter();
      const TileInfo ti = hooks.pairTileAt(s, t, groupRows, static_cast<int>(cta));
      const uint32_t tmemAcc = tmemBase + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kPairBN;
      epi.template operator()<kSpan>(tmemAcc, ti, s, laneRow, cBegin, rowStage);
      sm100::tcFenceBefore();
      __syncwarp();
      if (lane == 0) sm100::mbarArriveCluster(acc == 0 ? accEmptyFirst0 : accEmptyFirst1);
      if (++acc == 2) {
        acc = 0;
        accPhase ^= 1u;
      }
    }
    if (ok) hooks.afterTiles(hs, abortFlag);
  } else {
    // ---------------- extra warps (policy), both CTAs ----------------
    hooks.extraRole(hs, abortFlag);
  }

  __syncthreads();
  if (threadIdx.x == 0) {
    if (*abortFlag) {
      if (errorFlag) *reinterpret_cast<volatile int*>(errorFlag) = 1;  // may live in mapped host memory
    } else {
      hooks.teardown(hs);
    }
  }
  // No MMA of the pair is in flight and no CTA still signals the other.
  sm100::tcFenceBefore();
  sm100::clusterSync();
  sm100::tcFenceAfter();
  if (warp == 1) sm100::tmemDeallocPair(tmemBase, kTmemCols);
}

}  // namespace gemm
}  // namespace vccl
