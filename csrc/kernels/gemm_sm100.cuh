// SPDX-License-Identifier: Apache-2.0
// Persistent bf16 GEMM on 5th-generation tensor cores (sm_100a).
//
//   C[M, N] = A[M, K] * B[N, K]^T      (A, B K-major; fp32 accumulation)
//
// One CTA per SM loops over output tiles.  Warp roles:
//   warp 0     TMA producer: loads A and B k-blocks (128B swizzle) into a
//              STAGES-deep shared-memory ring, signalling `full` mbarriers.
//   warp 1     MMA issuer: one elected thread issues tcgen05.mma (M=128,
//              N=BN, K=16) into a TMEM accumulator, releasing ring slots
//              with tcgen05.commit -> `empty`.  Owns the TMEM allocation.
//   warps 2-5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM
//              lanes 32*(w%4)..+31 = tile rows), apply the Epilogue policy,
//              hand the accumulator back.  Two accumulators alternate so
//              the epilogue of tile i overlaps the MMAs of tile i+1.
//   warps 6+   optional extra warps run Policy::extraRole (used by the
//              all-gather + GEMM kernel to pull remote shards).
// The Policy decides the tile order, may gate a tile's loads on data
// arrival, and runs code before/after the epilogue's tiles; this is how the
// fused kernels reuse the mainloop.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "kernels/sm100.cuh"

namespace vccl {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle atom of bf16
// Threads of a CTA before the policy's extra warps: producer, MMA issuer and
// 4 x kEpiGroups epilogue warps.
template <typename Hooks>
__host__ __device__ constexpr int baseThreads() {
  return 64 + 128 * Hooks::kEpiGroups;
}
template <typename Hooks>
__host__ __device__ constexpr int ctaThreads() {
  return baseThreads<Hooks>() + 32 * Hooks::kExtraWarps;
}

constexpr int kWarpStageBytes = 32 * 8 * 16;  // epilogue row stage: 32 rows x 128 B per warp

template <int BN, int STAGES, int EPI_WARPS = 4>
struct Smem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kRowStageOff = STAGES * kStageBytes;
  static constexpr int kBarOff = kRowStageOff + EPI_WARPS * kWarpStageBytes;
  static constexpr int kBytes = kBarOff + 256 + 1024;  // + barriers + alignment slack
  static_assert(kBytes <= 232448, "shared memory budget of one CTA");
};

struct TileInfo {
  int tm, tn;    // tile coordinates
  int row0, col0;
  int ks;        // K split of this tile (0 without split-K)
  int kb0, kb1;  // k-blocks [kb0, kb1) accumulated into this tile
};

struct GemmShape {
  int M, N, K;
  int tilesM, tilesN;
  int splits;  // K splits (1: every tile covers all of K)
  // Rows of A the TMA box carries (a multiple of 8, at most kBM).  Decode
  // shapes load only their M rows instead of a zero-filled 128-row tile; the
  // MMA still reads 128 rows, and the accumulator rows past M are never
  // stored.
  int aRows;
  __host__ __device__ int numK() const { return (K + kBK - 1) / kBK; }
};

__device__ __forceinline__ uint32_t packBf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---- epilogue output path ------------------------------------------------------
// tcgen05.ld leaves one tile row per thread, so storing straight from
// registers makes every warp store instruction touch 32 different rows.
// Over NVLink that becomes 32 small write packets.  Instead each epilogue
// warp stages a 32-row x (NC x 16 B) slice in shared memory and writes it
// back row-contiguously: NC lanes per row, 32/NC rows per instruction, so a
// row segment of up to 128 B leaves as one request.  Chunks are XOR-swizzled
// by row so both the row-per-thread writes and the row-contiguous reads are
// free of bank conflicts.
// Slot of (row, chunk) in a warp's stage of 32 rows x NC 16-byte chunks.
__host__ __device__ constexpr int stageSlot(int nc, int row, int chunk) { return row * nc + (chunk ^ (row & (nc - 1))); }

template <int NC>
__device__ __forceinline__ void stagePut(uint4* st, int lane, int j, uint4 v) {
  st[stageSlot(NC, lane, j)] = v;
}

// dst(rowInWarp, chunk, value) is called for every staged 16-byte chunk.
template <int NC, typename Dst>
__device__ __forceinline__ void stageFlush(const uint4* st, int lane, Dst&& dst) {
  __syncwarp();
  constexpr int kRows = 32 / NC;
#pragma unroll
  for (int i = 0; i < NC; i++) {
    const int rr = i * kRows + lane / NC;
    const int ch = lane % NC;
    dst(rr, ch, st[stageSlot(NC, rr, ch)]);
  }
  __syncwarp();
}

__device__ __forceinline__ uint4 packChunk(const uint32_t* r) {
  uint4 o;
  o.x = packBf16(__uint_as_float(r[0]), __uint_as_float(r[1]));
  o.y = packBf16(__uint_as_float(r[2]), __uint_as_float(r[3]));
  o.z = packBf16(__uint_as_float(r[4]), __uint_as_float(r[5]));
  o.w = packBf16(__uint_as_float(r[6]), __uint_as_float(r[7]));
  return o;
}

// Write accumulator columns [cBegin, cBegin + SPAN) of the tile as bf16
// through the warp's row stage `st`.  rowBase(row) returns the byte address
// of column 0 of `row` (any memory this GPU can store to).  Columns are
// checked per 8-element chunk (N % 8 == 0).
template <int SPAN, typename RowBase>
__device__ __forceinline__ void storeAccRows(uint32_t tmemAcc, const TileInfo& ti, const GemmShape& s, int laneRow,
                                             int cBegin, uint4* st, RowBase&& rowBase) {
  constexpr int CW = SPAN < 64 ? SPAN : 64;  // accumulator columns per pass
  constexpr int NC = CW / 8;                 // 16-byte chunks per row per pass
  const int lane = laneRow & 31;
  const int warpRow0 = ti.row0 + (laneRow & ~31);
#pragma unroll 1
  for (int c = cBegin; c < cBegin + SPAN; c += CW) {
    uint32_t r[CW];
#pragma unroll
    for (int i = 0; i < CW / 16; i++) sm100::tmemLoad16p(tmemAcc + c + 16 * i, r + 16 * i);
    sm100::tmemLoadWait();
#pragma unroll
    for (int j = 0; j < NC; j++) stagePut<NC>(st, lane, j, packChunk(r + 8 * j));
    const int col0 = ti.col0 + c;
    stageFlush<NC>(st, lane, [&](int rr, int ch, uint4 v) {
      const int row = warpRow0 + rr, col = col0 + ch * 8;
      if (row < s.M && col < s.N) *reinterpret_cast<uint4*>(rowBase(row) + static_cast<size_t>(col) * 2) = v;
    });
  }
}

// Plain store of the accumulator to C (row-major, ldc elements).
// Every epilogue functor writes accumulator columns [cBegin, cBegin + SPAN)
// of the tile rows owned by the calling thread's warp.
struct EpiStore {
  __nv_bfloat16* C;
  int ldc;
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const TileInfo& ti, const GemmShape& s, int laneRow,
                                             int cBegin, uint4* st) const {
    char* base = reinterpret_cast<char*>(C);
    const size_t pitch = static_cast<size_t>(ldc) * 2;
    storeAccRows<SPAN>(tmemAcc, ti, s, laneRow, cBegin, st, [&](int row) { return base + row * pitch; });
  }
};

// Split-K partial: writes the fp32 accumulator of split ti.ks to
// ws[ks][row][col] (row-major, ldn columns); a reduction kernel sums the
// splits.  Rows leave as 128-byte segments (32 floats).
struct EpiPartialF32 {
  float* ws;
  int ldn;
  size_t splitElems;  // elements per split slice (M * ldn)
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const TileInfo& ti, const GemmShape& s, int laneRow,
                                             int cBegin, uint4* st) const {
    constexpr int CW = SPAN < 32 ? SPAN : 32;  // accumulator columns per pass
    constexpr int NC = CW / 4;                 // 16-byte chunks per row per pass
    const int lane = laneRow & 31;
    const int warpRow0 = ti.row0 + (laneRow & ~31);
    float* base = ws + static_cast<size_t>(ti.ks) * splitElems;
#pragma unroll 1
    for (int c = cBegin; c < cBegin + SPAN; c += CW) {
      uint32_t r[CW];
#pragma unroll
      for (int i = 0; i < CW / 16; i++) sm100::tmemLoad16p(tmemAcc + c + 16 * i, r + 16 * i);
      sm100::tmemLoadWait();
#pragma unroll
      for (int j = 0; j < NC; j++) stagePut<NC>(st, lane, j, make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]));
      const int col0 = ti.col0 + c;
      stageFlush<NC>(st, lane, [&](int rr, int ch, uint4 v) {
        const int row = warpRow0 + rr, col = col0 + ch * 4;
        if (row < s.M && col < s.N)
          *reinterpret_cast<uint4*>(base + static_cast<size_t>(row) * ldn + col) = v;
      });
    }
  }
};

// Split-K with the reduction inside the GEMM, for decode shapes (a few
// rows, so a tile's fix-up is a short job for one warp).  Every split stores its
// fp32 partial as EpiPartialF32 does; then each epilogue warp that holds
// valid rows counts itself on the (tile, lane quarter) semaphore, and the
// warp of the split that arrives last sums those rows' partials in split
// order (the order of the separate reduction kernel, so the results are the
// same bits) and writes bf16 C, or silu(gate) * up for the interleaved
// gate/up layout of EpiSiluMul.  This saves the reduction kernel's launch
// and its pass over the partials.  Only warp-level synchronisation is used.
// The semaphores are zero before a call and the last arriver puts its
// semaphore back to zero.  One epilogue warpgroup only (NoHooks);
// `afterTile` runs once the accumulator has been handed back, so the fix-up
// overlaps the next tile's MMAs.
template <bool SILU>
struct EpiSplitFixup {
  static constexpr bool kAfterTile = true;
  EpiPartialF32 part;
  uint32_t* sem;      // [tilesM * tilesN][4]: per output tile and TMEM lane quarter
  __nv_bfloat16* C;   // [M, N] (or [M, N / 2] with SILU)
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const TileInfo& ti, const GemmShape& s, int laneRow,
                                             int cBegin, uint4* st) const {
    part.template operator()<SPAN>(tmemAcc, ti, s, laneRow, cBegin, st);
  }
  // One epilogue warp: `quarter` is its TMEM lane quarter (tile rows
  // 32 * quarter ... + 31), `lane` its lane.
  template <int BN>
  __device__ __forceinline__ void afterTile(const TileInfo& ti, const GemmShape& s, int quarter, int lane) const {
    const int r0 = ti.row0 + 32 * quarter;
    if (r0 >= s.M) return;  // no valid rows: this warp stored nothing and counts nothing
    const int rows = s.M - r0 < 32 ? s.M - r0 : 32;
    __syncwarp();  // every lane's partial stores are issued
    uint32_t last = 0;
    if (lane == 0) {
      __threadfence();  // ... and visible device-wide before the count
      uint32_t* cnt = sem + (ti.tm * s.tilesN + ti.tn) * 4 + quarter;
      last = atomicAdd(cnt, 1u) == static_cast<uint32_t>(s.splits - 1) ? 1u : 0u;
      if (last) {
        *cnt = 0u;        // every split of this call has counted: ready for the next call
        __threadfence();  // order the other splits' partials before the loads below
      }
    }
    if (__shfl_sync(0xffffffffu, last, 0) == 0u) return;
    __syncwarp();  // lane 0's acquire (the fence after the count) orders the whole warp's loads
    const size_t ldn = static_cast<size_t>(part.ldn);
    const float* base = part.ws + static_cast<size_t>(r0) * ldn;
    if constexpr (!SILU) {
      constexpr int G = BN / 4;  // float4 groups per tile row
      for (int idx = lane; idx < rows * G; idx += 32) {
        const int r = idx / G;
        const int col = ti.col0 + 4 * (idx - r * G);
        if (col >= s.N) continue;
        const float* p = base + r * ldn + col;
        float4 a = __ldcg(reinterpret_cast<const float4*>(p));
        for (int k = 1; k < s.splits; k++) {
          const float4 b = __ldcg(reinterpret_cast<const float4*>(p + k * part.splitElems));
          a.x += b.x;
          a.y += b.y;
          a.z += b.z;
          a.w += b.w;
        }
        *reinterpret_cast<uint2*>(C + static_cast<size_t>(r0 + r) * s.N + col) =
            make_uint2(packBf16(a.x, a.y), packBf16(a.z, a.w));
      }
    } else {
      constexpr int G = BN / 8;  // groups of 4 outputs per tile row (BN / 2 outputs)
      const int half = s.N / 2;
      for (int idx = lane; idx < rows * G; idx += 32) {
        const int r = idx / G;
        const int jl = 4 * (idx - r * G);  // output column inside the tile
        const int gcol = ti.col0 + (jl / 16) * 32 + (jl % 16);
        const int j = ti.col0 / 2 + jl;    // output column
        if (j >= half) continue;
        const float* p = base + r * ldn + gcol;
        float4 g = __ldcg(reinterpret_cast<const float4*>(p));
        float4 u = __ldcg(reinterpret_cast<const float4*>(p + 16));
        for (int k = 1; k < s.splits; k++) {
          const float4 g2 = __ldcg(reinterpret_cast<const float4*>(p + k * part.splitElems));
          const float4 u2 = __ldcg(reinterpret_cast<const float4*>(p + k * part.splitElems + 16));
          g.x += g2.x, g.y += g2.y, g.z += g2.z, g.w += g2.w;
          u.x += u2.x, u.y += u2.y, u.z += u2.z, u.w += u2.w;
        }
        auto f = [](float x, float y) { return x / (1.0f + __expf(-x)) * y; };
        *reinterpret_cast<uint2*>(C + static_cast<size_t>(r0 + r) * half + j) =
            make_uint2(packBf16(f(g.x, u.x), f(g.y, u.y)), packBf16(f(g.z, u.z), f(g.w, u.w)));
      }
    }
  }
};

template <typename E, typename = void>
struct HasAfterTile {
  static constexpr bool value = false;
};
template <typename E>
struct HasAfterTile<E, decltype((void)E::kAfterTile)> {
  static constexpr bool value = E::kAfterTile;
};

// Gate/up epilogue.  B holds the gate and up projections interleaved in
// groups of 16 rows (g0..15, u0..15, g16..31, u16..31, ...), so every
// 32-column slice of the accumulator is (16 gate, 16 up) of the same output
// columns for any tile width.  Writes silu(gate) * up; C has N/2 columns.
struct EpiSiluMul {
  __nv_bfloat16* C;
  int ldc;
  template <int SPAN>
  __device__ __forceinline__ void operator()(uint32_t tmemAcc, const TileInfo& ti, const GemmShape& s, int laneRow,
                                             int cBegin, uint4* st) const {
    static_assert(SPAN % 32 == 0, "gate/up pairs span 32 accumulator columns");
    constexpr int CW = SPAN < 128 ? SPAN : 128;  // accumulator columns per pass
    constexpr int NC = CW / 16;                  // 16-byte output chunks per row per pass
    const int lane = laneRow & 31;
    const int warpRow0 = ti.row0 + (laneRow & ~31);
    char* base = reinterpret_cast<char*>(C);
    const size_t pitch = static_cast<size_t>(ldc) * 2;
#pragma unroll 1
    for (int c = cBegin; c < cBegin + SPAN; c += CW) {
#pragma unroll
      for (int j = 0; j < CW / 32; j++) {
        uint32_t g[16], u[16];
        sm100::tmemLoad16(tmemAcc + c + 32 * j, g);
        sm100::tmemLoad16(tmemAcc + c + 32 * j + 16, u);
        sm100::tmemLoadWait();
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float x0 = __uint_as_float(g[2 * i]), x1 = __uint_as_float(g[2 * i + 1]);
          o[i] = packBf16(x0 / (1.0f + __expf(-x0)) * __uint_as_float(u[2 * i]),
                          x1 / (1.0f + __expf(-x1)) * __uint_as_float(u[2 * i + 1]));
        }
        stagePut<NC>(st, lane, 2 * j, make_uint4(o[0], o[1], o[2], o[3]));
        stagePut<NC>(st, lane, 2 * j + 1, make_uint4(o[4], o[5], o[6], o[7]));
      }
      const int col0 = (ti.col0 + c) / 2;
      stageFlush<NC>(st, lane, [&](int rr, int ch, uint4 v) {
        const int row = warpRow0 + rr, col = col0 + ch * 8;
        if (row < s.M && col < s.N / 2) *reinterpret_cast<uint4*>(base + row * pitch + static_cast<size_t>(col) * 2) = v;
      });
    }
  }
};

// Tile orders (host and device, so CPU tests can check them).
//
// splitKTile: N-major order (consecutive CTAs share the B tile); with
// split-K, tile t covers output tile t % (tilesM * tilesN) over the k-blocks
// of split t / (tilesM * tilesN).
__host__ __device__ inline TileInfo splitKTile(const GemmShape& s, int t, int BN) {
  TileInfo ti;
  const int mn = s.tilesM * s.tilesN;
  ti.ks = t / mn;
  const int r = t - ti.ks * mn;
  ti.tn = r / s.tilesM;
  ti.tm = r % s.tilesM;
  ti.row0 = ti.tm * kBM;
  ti.col0 = ti.tn * BN;
  const int nk = s.numK();
  ti.kb0 = ti.ks * nk / s.splits;
  ti.kb1 = (ti.ks + 1) * nk / s.splits;
  return ti;
}

// groupedTile: row tiles start at startTm and wrap around; they are walked
// in groups of groupRows row tiles, and inside a group consecutive tiles
// share a column tile, so a wave of CTAs reads each B tile once per group.
__host__ __device__ inline TileInfo groupedTile(const GemmShape& s, int t, int BN, int groupRows, int startTm) {
  TileInfo ti;
  const int groupTiles = groupRows * s.tilesN;
  const int g = t / groupTiles;
  const int rowsHere = s.tilesM - g * groupRows < groupRows ? s.tilesM - g * groupRows : groupRows;
  const int local = t - g * groupTiles;
  ti.tn = local / rowsHere;
  ti.tm = (g * groupRows + local % rowsHere + startTm) % s.tilesM;
  ti.row0 = ti.tm * kBM;
  ti.col0 = ti.tn * BN;
  ti.ks = 0;
  ti.kb0 = 0;
  ti.kb1 = s.numK();
  return ti;
}

// Default policy: tiles in N-major order (consecutive CTAs share the B
// tile), no gating, no extra warps.  `hs` is per-CTA shared scratch.
struct NoHooks {
  static constexpr int kExtraWarps = 0;
  static constexpr int kEpiGroups = 1;  // epilogue warpgroups; each takes BN / kEpiGroups columns
  __device__ __forceinline__ void setup(uint32_t*) const {}
  __device__ __forceinline__ void teardown(uint32_t*) const {}
  // With split-K, tile t covers output tile t % (tilesM * tilesN) over the
  // k-blocks of split t / (tilesM * tilesN).
  __device__ __forceinline__ TileInfo tileAt(const GemmShape& s, int t, int BN) const {
    return splitKTile(s, t, BN);
  }
  __device__ __forceinline__ bool beforeLoad(const TileInfo&, const GemmShape&, uint32_t*, volatile int*) const {
    return true;
  }
  __device__ __forceinline__ bool beforeTiles(uint32_t*, volatile int*) const { return true; }
  __device__ __forceinline__ void afterTiles(uint32_t*, volatile int*) const {}
  __device__ __forceinline__ void extraRole(uint32_t*, volatile int*) const {}
};

template <int BN, int STAGES, typename Epi, typename Hooks = NoHooks>
__global__ void __launch_bounds__(ctaThreads<Hooks>(), 1)
    gemmKernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, GemmShape s,
               const __grid_constant__ Epi epi, Hooks hooks, int* errorFlag) {
  constexpr int kEpiWarps = 4 * Hooks::kEpiGroups;
  constexpr int kSpan = BN / Hooks::kEpiGroups;
  using L = Smem<BN, STAGES, kEpiWarps>;
  extern __shared__ __align__(1024) uint8_t smemRaw[];
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
  constexpr uint32_t kTmemCols = 2 * BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; i++) {
      sm100::mbarInit(&fullBar[i], 1);
      sm100::mbarInit(&emptyBar[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      sm100::mbarInit(&accFull[i], 1);
      sm100::mbarInit(&accEmpty[i], kEpiWarps);
    }
    sm100::mbarInit(drainBar, 1);
    *abortFlag = 0;
    hooks.setup(hs);
    sm100::fenceBarrierInit();
  }
  if (warp == 1) {
    sm100::tmemAlloc(tmemSlot, kTmemCols);
    sm100::tmemRelinquish();
  }
  sm100::tcFenceBefore();
  __syncthreads();
  sm100::tcFenceAfter();
  const uint32_t tmemBase = *tmemSlot;
  const int numTiles = s.tilesM * s.tilesN * s.splits;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (sm100::electOne()) {
      sm100::tmaPrefetchDesc(&mapA);
      sm100::tmaPrefetchDesc(&mapB);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < numTiles && ok; t += gridDim.x) {
        const TileInfo ti = hooks.tileAt(s, t, BN);
        if (!hooks.beforeLoad(ti, s, hs, abortFlag)) {
          *abortFlag = 1;
          ok = false;
          break;
        }
        for (int kb = ti.kb0; kb < ti.kb1; kb++) {
          if (!sm100::mbarWait(&emptyBar[stage], phase ^ 1u, abortFlag)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + stage * L::kStageBytes;
          uint8_t* b = a + L::kABytes;
          sm100::mbarArriveExpectTx(&fullBar[stage], static_cast<uint32_t>(s.aRows * kBK * 2 + L::kBBytes));
          sm100::tmaLoad2d(a, &mapA, &fullBar[stage], kb * kBK, ti.row0);
          sm100::tmaLoad2d(b, &mapB, &fullBar[stage], kb * kBK, ti.col0);
          issued++;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA can exit.
        const int n = issued < static_cast<uint32_t>(STAGES) ? static_cast<int>(issued) : STAGES;
        int s2 = stage;
        uint32_t p2 = phase;
        for (int i = 0; i < n; i++) {
          if (--s2 < 0) {
            s2 = STAGES - 1;
            p2 ^= 1u;
          }
          volatile int never = 0;
          sm100::mbarWait(&fullBar[s2], p2, &never, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (sm100::electOne()) {
      constexpr uint32_t idesc = sm100::idescBf16F32(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t accPhase = 0;
      bool ok = true;
      bool anyIssued = false;
      for (int t = blockIdx.x; t < numTiles && ok; t += gridDim.x) {
        if (!sm100::mbarWait(&accEmpty[acc], accPhase ^ 1u, abortFlag)) {
          ok = false;
          break;
        }
        sm100::tcFenceAfter();
        const uint32_t tmemAcc = tmemBase + acc * BN;
        const TileInfo ti = hooks.tileAt(s, t, BN);
        for (int kb = ti.kb0; kb < ti.kb1; kb++) {
          if (!sm100::mbarWait(&fullBar[stage], phase, abortFlag)) {
            ok = false;
            break;
          }
          sm100::tcFenceAfter();
          const uint32_t aAddr = sm100::smemAddr(smem + stage * L::kStageBytes);
          const uint32_t bAddr = aAddr + L::kABytes;
          const uint64_t ad = sm100::smemDescSw128(aAddr);
          const uint64_t bd = sm100::smemDescSw128(bAddr);
#pragma unroll
          for (int k = 0; k < kBK / 16; k++) {
            // +32 bytes per K=16 step inside the swizzle atom (descriptor units of 16 B).
            sm100::mmaBf16(tmemAcc, ad + 2 * k, bd + 2 * k, idesc, (kb != ti.kb0 || k != 0) ? 1u : 0u);
          }
          anyIssued = true;
          sm100::mmaCommit(&emptyBar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        sm100::mmaCommit(&accFull[acc]);
        if (++acc == 2) {
          acc = 0;
          accPhase ^= 1u;
        }
      }
      if (!ok && anyIssued) {
        // Drain every MMA in flight before TMEM is released.
        sm100::mmaCommit(drainBar);
        volatile int never = 0;
        sm100::mbarWait(drainBar, 0, &never, 200000000ull);
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ---------------- epilogue (warps 2 .. 1 + kEpiWarps) ----------------
    const int quarter = warp & 3;             // TMEM lane quarter this warp may access
    const int laneRow = quarter * 32 + lane;  // tile row of this thread
    const int cBegin = ((warp - 2) / 4) * kSpan;
    uint4* rowStage = reinterpret_cast<uint4*>(smem + L::kRowStageOff + (warp - 2) * kWarpStageBytes);
    int acc = 0;
    uint32_t accPhase = 0;
    bool ok = hooks.beforeTiles(hs, abortFlag);
    if (!ok) *abortFlag = 1;
    for (int t = blockIdx.x; t < numTiles && ok; t += gridDim.x) {
      if (!sm100::mbarWait(&accFull[acc], accPhase, abortFlag)) {
        ok = false;
        break;
      }
      sm100::tcFenceAfter();
      const TileInfo ti = hooks.tileAt(s, t, BN);
      const uint32_t tmemAcc = tmemBase + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      epi.template operator()<kSpan>(tmemAcc, ti, s, laneRow, cBegin, rowStage);
      sm100::tcFenceBefore();
      __syncwarp();
      if (lane == 0) sm100::mbarArrive(&accEmpty[acc]);
      if constexpr (HasAfterTile<Epi>::value) epi.template afterTile<BN>(ti, s, quarter, lane);
      if (++acc == 2) {
        acc = 0;
        accPhase ^= 1u;
      }
    }
    if (ok) hooks.afterTiles(hs, abortFlag);
  } else {
    // ---------------- extra warps (policy) ----------------
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
  if (warp == 1) {
    sm100::tcFenceAfter();
    sm100::tmemDealloc(tmemBase, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace vccl
