// SPDX-License-Identifier: Apache-2.0
// Index arithmetic of the GEMM kernels, checked on the host (no GPU):
//  * splitKTile visits every (row tile, column tile, K split) exactly once and
//    the K splits of a tile partition its k-blocks;
//  * groupedTile (all-gather + GEMM order) is a permutation of the tiles for
//    every shard rotation, and starts with the first rank-owned row tile;
//  * the epilogue row stage: every (row, chunk) has its own slot, and each
//    8-lane phase of both the row-per-thread writes and the row-contiguous
//    reads touches 8 different 16-byte bank groups;
//  * pairTile (CTA-pair GEMM order) visits every 256 x 256 tile once for
//    every grouping, and the two CTAs of a pair take its two 128-row halves;
//  * planSplitK keeps its bounds (4+ k-blocks per split, <= 16 splits,
//    partials <= a quarter of the weight bytes).
#include <cstdio>
#include <cstdlib>
#include <set>
#include <tuple>
#include <vector>

#include "fused/gemm_host.h"
#include "kernels/gemm_sm100.cuh"
#include "kernels/gemm_sm100_pair.cuh"

using namespace vccl::gemm;

namespace {
int gFail = 0;
#define EXPECT(c, ...)                                          \
  do {                                                          \
    if (!(c)) {                                                 \
      std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      std::fprintf(stderr, __VA_ARGS__);                        \
      std::fprintf(stderr, "\n");                               \
      gFail++;                                                  \
    }                                                           \
  } while (0)

GemmShape shape(int M, int N, int K, int BN, int splits) {
  GemmShape s{};
  s.M = M;
  s.N = N;
  s.K = K;
  s.tilesM = (M + kBM - 1) / kBM;
  s.tilesN = (N + BN - 1) / BN;
  s.splits = splits;
  s.aRows = M >= kBM ? kBM : (M + 7) / 8 * 8;
  return s;
}

void checkPairTiles() {
  for (int M : {256, 1000, 8192})
    for (int N : {256, 1040, 28672})
      for (int group : {1, 3, 8, 64}) {
        GemmShape s{};
        s.M = M;
        s.N = N;
        s.K = 4096;
        s.tilesM = (M + kPairBM - 1) / kPairBM;
        s.tilesN = (N + kPairBN - 1) / kPairBN;
        s.splits = 1;
        s.aRows = kBM;
        std::set<std::pair<int, int>> seen;
        for (int t = 0; t < s.tilesM * s.tilesN; t++) {
          const TileInfo t0 = pairTile(s, t, group, 0), t1 = pairTile(s, t, group, 1);
          EXPECT(t0.tm >= 0 && t0.tm < s.tilesM && t0.tn >= 0 && t0.tn < s.tilesN, "pair tile out of range");
          EXPECT(seen.insert({t0.tm, t0.tn}).second, "pair tile visited twice (M=%d N=%d group=%d)", M, N, group);
          EXPECT(t0.tm == t1.tm && t0.tn == t1.tn, "the CTAs of a pair disagree on the tile");
          EXPECT(t0.row0 == t0.tm * kPairBM && t1.row0 == t0.row0 + kBM, "pair row halves");
          EXPECT(t0.col0 == t0.tn * kPairBN && t1.col0 == t0.col0, "pair columns");
          EXPECT(t0.kb0 == 0 && t0.kb1 == s.numK(), "pair tiles cover all of K");
        }
        EXPECT(static_cast<int>(seen.size()) == s.tilesM * s.tilesN, "pair tiles missing");
        // split-K on pairs: every (tile, split) once, the splits partition the k-blocks
        for (int splits : {2, 3, 4}) {
          s.splits = splits;
          std::vector<int> cover(static_cast<size_t>(s.tilesM) * s.tilesN * s.numK(), 0);
          for (int t = 0; t < s.tilesM * s.tilesN * splits; t++) {
            const TileInfo ti = pairTile(s, t, group, 0);
            EXPECT(ti.kb0 < ti.kb1 && ti.ks == t / (s.tilesM * s.tilesN), "pair split range");
            for (int kb = ti.kb0; kb < ti.kb1; kb++)
              cover[(static_cast<size_t>(ti.tm) * s.tilesN + ti.tn) * s.numK() + kb]++;
          }
          bool once = true;
          for (int c : cover) once = once && c == 1;
          EXPECT(once, "pair split-K covers a k-block twice or not at all (M=%d N=%d splits=%d)", M, N, splits);
          s.splits = 1;
        }
      }
}

void checkSplitK() {
  for (int M : {1, 100, 128, 300, 1024})
    for (int N : {32, 512, 3584})
      for (int K : {64, 1000, 4096})
        for (int BN : {32, 64, 128, 256})
          for (int splits : {1, 2, 3, 5, 16}) {
            GemmShape s = shape(M, N, K, BN, splits);
            if (splits > s.numK()) continue;
            std::vector<int> kbCover(static_cast<size_t>(s.tilesM) * s.tilesN * s.numK(), 0);
            std::set<std::tuple<int, int, int>> seen;
            for (int t = 0; t < s.tilesM * s.tilesN * splits; t++) {
              TileInfo ti = splitKTile(s, t, BN);
              EXPECT(seen.insert({ti.tm, ti.tn, ti.ks}).second, "tile visited twice");
              EXPECT(ti.row0 == ti.tm * kBM && ti.col0 == ti.tn * BN, "tile origin");
              EXPECT(ti.kb0 < ti.kb1, "empty K range (M=%d N=%d K=%d splits=%d)", M, N, K, splits);
              for (int kb = ti.kb0; kb < ti.kb1; kb++)
                kbCover[(static_cast<size_t>(ti.tm) * s.tilesN + ti.tn) * s.numK() + kb]++;
            }
            for (int c : kbCover) EXPECT(c == 1, "k-block covered %d times", c);
          }
}

void checkGrouped() {
  for (int ranks : {1, 2, 4, 8})
    for (int shardTiles : {1, 2, 3, 8, 16})
      for (int N : {256, 3584, 7168}) {
        const int M = ranks * shardTiles * kBM;
        GemmShape s = shape(M, N, 4096, 256, 1);
        int groupRows = 1;
        for (int g = 16; g >= 1; g /= 2)
          if (shardTiles % g == 0) {
            groupRows = g;
            break;
          }
        for (int r = 0; r < ranks; r++) {
          const int startTm = r * shardTiles;
          std::set<std::pair<int, int>> seen;
          for (int t = 0; t < s.tilesM * s.tilesN; t++) {
            TileInfo ti = groupedTile(s, t, 256, groupRows, startTm);
            EXPECT(ti.tm >= 0 && ti.tm < s.tilesM && ti.tn >= 0 && ti.tn < s.tilesN, "tile out of range");
            EXPECT(seen.insert({ti.tm, ti.tn}).second, "grouped tile visited twice");
            EXPECT(ti.kb0 == 0 && ti.kb1 == s.numK(), "grouped tiles cover all of K");
          }
          EXPECT(static_cast<int>(seen.size()) == s.tilesM * s.tilesN, "grouped order misses tiles");
          EXPECT(groupedTile(s, 0, 256, groupRows, startTm).tm == startTm, "first tile is the own shard's");
        }
      }
}

void checkStage() {
  for (int nc : {2, 4, 8}) {
    std::set<int> slots;
    for (int row = 0; row < 32; row++)
      for (int ch = 0; ch < nc; ch++) {
        const int sl = stageSlot(nc, row, ch);
        EXPECT(sl >= 0 && sl < 32 * nc && slots.insert(sl).second, "stage slot collision (nc=%d)", nc);
      }
    // With 8 chunks (128-byte rows) the stage is the layout a TMA tile store
    // with 128-byte swizzle reads from a 1024-byte aligned box: byte address
    // bits [4,7) are XORed with bits [7,10).
    if (nc == 8)
      for (int row = 0; row < 32; row++)
        for (int ch = 0; ch < 8; ch++) {
          const int plain = row * 128 + ch * 16;
          const int swz = plain ^ (((plain >> 7) & 7) << 4);
          EXPECT(stageSlot(8, row, ch) * 16 == swz, "stage differs from the 128-byte swizzle at row %d chunk %d",
                 row, ch);
        }
    // writes: lane = row, one instruction per chunk j; phases of 8 lanes
    for (int j = 0; j < nc; j++)
      for (int ph = 0; ph < 4; ph++) {
        std::set<int> banks;
        for (int l = ph * 8; l < ph * 8 + 8; l++) banks.insert(stageSlot(nc, l, j) % 8);
        if (nc == 8) EXPECT(banks.size() == 8, "write phase bank conflict");
      }
    // reads: instruction i, lane -> (row i*(32/nc) + lane/nc, chunk lane%nc)
    const int rows = 32 / nc;
    for (int i = 0; i < nc; i++)
      for (int ph = 0; ph < 4; ph++) {
        std::set<int> banks;
        for (int l = ph * 8; l < ph * 8 + 8; l++) banks.insert(stageSlot(nc, i * rows + l / nc, l % nc) % 8);
        if (nc == 8) EXPECT(banks.size() == 8, "read phase bank conflict");
      }
  }
}

void checkPlan() {
  for (int M : {1, 16, 32, 64, 128, 200, 256, 300})
    for (int N : {512, 1536, 3584, 8192, 28672})
      for (int K : {256, 1792, 4096, 8192, 14336}) {
        SplitPlan p = planSplitK(M, N, K);
        const int numK = (K + kBK - 1) / kBK;
        if (p.splits <= 1) continue;
        EXPECT((M + kBM - 1) / kBM <= 2, "split-K only for decode shapes");
        EXPECT(p.splits <= 16 && numK / p.splits >= 4, "split bounds M=%d N=%d K=%d s=%d", M, N, K, p.splits);
        EXPECT(static_cast<double>(M) * N * p.splits * 4 <= static_cast<double>(N) * K * 2 / 4 + 1,
               "partials above a quarter of the weights (M=%d N=%d K=%d s=%d)", M, N, K, p.splits);
        EXPECT(p.bn == 128, "split-K tile width");
      }
}
// CTA-pair plans on a 148-SM device with 74 pairs: the large bench shapes run
// on pairs without splitting K; a shape with too few pair tiles to fill the
// device (512 x 4096 x 14336: 32 tiles) splits K in two; a shape smaller
// than one pair tile never takes the pair kernel; VCCL_GEMM_PAIR=0 turns
// pairs off (the plan reads the variable per call).
void checkPairPlan() {
  unsetenv("VCCL_GEMM_PAIR");
  PairPlan p = planPair(8192, 28672, 4096, 0, 74);
  EXPECT(p.use && p.splits == 1, "8192x28672x4096: use=%d splits=%d", p.use, p.splits);
  p = planPair(8192, 4096, 14336, 0, 74);
  EXPECT(p.use && p.splits == 1, "8192x4096x14336: use=%d splits=%d", p.use, p.splits);
  p = planPair(512, 4096, 14336, 0, 74);
  EXPECT(p.use && p.splits == 2, "512x4096x14336: use=%d splits=%d", p.use, p.splits);
  p = planPair(128, 4096, 4096, 0, 74);
  EXPECT(!p.use, "M below one pair tile");
  p = planPair(8192, 4096, 4096, 64, 74);
  EXPECT(!p.use, "a tile-width override keeps one-SM tiles");
  for (int M : {256, 512, 1000, 4096, 8192})
    for (int N : {256, 1024, 4096, 28672})
      for (int K : {512, 4096, 14336}) {
        p = planPair(M, N, K, 0, 74);
        const int nk = (K + kBK - 1) / kBK;
        EXPECT(p.splits >= 1 && p.splits <= 4 && (p.splits == 1 || nk / p.splits >= 8),
               "pair split bounds M=%d N=%d K=%d s=%d", M, N, K, p.splits);
      }
  setenv("VCCL_GEMM_PAIR", "0", 1);
  EXPECT(!planPair(8192, 28672, 4096, 0, 74).use, "VCCL_GEMM_PAIR=0");
  unsetenv("VCCL_GEMM_PAIR");
}

// Makespan tile widths: the TP-8 gate/up shard (896 tiles at 256 = 6.05
// waves) goes to 128; full-wave shapes stay at 256; a 512-row GEMM takes one
// wave of 128-wide tiles instead of two of 64; one-wave decode shapes take
// the narrowest tile.
void checkPickWaves() {
  EXPECT(pickBNWaves(8192, 3584, 148) == 128, "8192x3584 -> %d", pickBNWaves(8192, 3584, 148));
  EXPECT(pickBNWaves(8192, 4096, 148) == 256, "8192x4096 -> %d", pickBNWaves(8192, 4096, 148));
  EXPECT(pickBNWaves(8192, 28672, 148) == 256, "8192x28672 -> %d", pickBNWaves(8192, 28672, 148));
  EXPECT(pickBNWaves(512, 3584, 148) == 128, "512x3584 -> %d", pickBNWaves(512, 3584, 148));
  EXPECT(pickBNWaves(1, 512, 148) == 32, "1x512 -> %d", pickBNWaves(1, 512, 148));
  for (int M : {1, 128, 1000, 8192})
    for (int N : {256, 1024, 3584, 4096, 14336})
      for (int sms : {132, 148}) {
        const int bn = pickBNWaves(M, N, sms);
        EXPECT(bn == 256 || bn == 128 || bn == 64 || bn == 32, "width %d", bn);
      }
}
}  // namespace

int main() {
  checkSplitK();
  checkPairTiles();
  checkPairPlan();
  checkPickWaves();
  checkGrouped();
  checkStage();
  checkPlan();
  std::printf("tiling: %s\n", gFail == 0 ? "OK" : "FAIL");
  return gFail == 0 ? 0 : 1;
}
