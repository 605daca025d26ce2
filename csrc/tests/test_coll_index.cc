// SPDX-License-Identifier: Apache-2.0
// Index arithmetic of the staged and zero-copy collective kernels, checked
// on the host (no GPU).  Each check restates a kernel's loops over blocks,
// rounds, pieces and rank chunks with the same split helpers the kernel
// calls (kernels/ranges.cuh, and the launcher's pipelined-NVLS geometry) and
// verifies that
//  * every byte (element) of the message is copied in, reduced and copied
//    out exactly once per rank, for any size, rank count and grid;
//  * every staging access stays inside the staging region, and inside the
//    block's own bytes of it, in every round (the property a re-split of a
//    short last round would break);
//  * the zero-copy window kernels partition each rank's chunk, and the
//    vector/tail split of a range covers it exactly;
//  * the split-K fix-up's SiLU*mul column mapping equals the reduction
//    kernel's.
#include <cstdio>
#include <cstring>
#include <map>
#include <vector>

#include "kernels/device_common.cuh"
#include "kernels/ranges.cuh"
#include "runtime/launch.h"

using namespace vccl;
using namespace vccl::dev;

namespace {
int gFail = 0;
#define EXPECT(c, ...)                                          \
  do {                                                          \
    if (!(c)) {                                                 \
      std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      std::fprintf(stderr, __VA_ARGS__);                        \
      std::fprintf(stderr, "\n");                               \
      if (++gFail > 20) return;                                 \
    }                                                           \
  } while (0)

// Staged NVLS all-reduce (allReduceNvls): rounds of n chunks of cb bytes.
void checkNvlsRounds(size_t total, int n, int G, size_t dataBytes) {
  const size_t roundBytes = (dataBytes - 16 * kMaxRanks) / 16 * 16;
  const size_t cb = nvlsRoundChunk(total, n, roundBytes);
  const size_t step = cb * n;
  EXPECT(cb % 16 == 0 && cb > 0, "chunk %zu", cb);
  EXPECT(step <= dataBytes, "round of %zu bytes exceeds staging %zu", step, dataBytes);
  std::vector<unsigned char> in(total, 0), red(total, 0), out(total, 0);
  std::vector<int> owner(step, -1);  // staging byte -> block that uses it
  for (size_t off = 0; off < total; off += step) {
    const size_t m = (total - off) < step ? (total - off) : step;
    for (int blk = 0; blk < G; blk++) {
      size_t s0, s1;
      blockRange(cb, G, blk, 16, &s0, &s1);
      for (int q = 0; q < n; q++) {
        const size_t lo = q * cb + s0, hiRaw = q * cb + s1, hi = hiRaw < m ? hiRaw : m;
        for (size_t b = lo; b < hi; b++) {
          in[off + b]++;
          out[off + b]++;
          EXPECT(owner[b] == -1 || owner[b] == blk, "staging byte %zu used by blocks %d and %d", b, owner[b], blk);
          owner[b] = blk;
        }
        // the owner of chunk q reduces it, 16-byte units rounded up inside the block's bytes
        if (lo < hi) {
          const size_t units = (hi - lo + 15) / 16;
          EXPECT(lo + units * 16 <= q * cb + s1, "reduce of chunk %d block %d leaves its bytes", q, blk);
          for (size_t b = lo; b < hi; b++) red[off + b]++;
        }
      }
    }
  }
  for (size_t b = 0; b < total; b++)
    EXPECT(in[b] == 1 && red[b] == 1 && out[b] == 1, "NVLS total=%zu n=%d G=%d byte %zu: in %d red %d out %d",
           total, n, G, b, in[b], red[b], out[b]);
}

// Two-shot all-reduce (allReduceTwoShot): rounds of n chunks of ce
// elements; block b pushes [s0, s1) of chunk q into slot `me` of rank q at
// the same chunk-relative offsets in every round.
void checkTwoShot(size_t count, int n, int G, size_t slotElems, size_t pk) {
  const size_t roundElems = slotElems * n;
  const size_t first = count < roundElems ? count : roundElems;
  const size_t ce = rankChunk(first, n, pk);
  EXPECT(ce <= slotElems, "chunk %zu exceeds the slot %zu", ce, slotElems);
  std::vector<unsigned char> done(count, 0);
  for (size_t base = 0; base < count; base += roundElems) {
    const size_t m = (count - base) < roundElems ? (count - base) : roundElems;
    for (int blk = 0; blk < G; blk++) {
      size_t s0, s1;
      blockRange(ce, G, blk, pk, &s0, &s1);
      for (int q = 0; q < n; q++) {
        const size_t lo = q * ce + s0, hiRaw = q * ce + s1, hi = hiRaw < m ? hiRaw : m;
        for (size_t e = lo; e < hi; e++) done[base + e]++;
        if (lo < hi) EXPECT(s0 + (hi - lo) <= s1 && s1 <= slotElems, "slot range of block %d", blk);
      }
    }
  }
  for (size_t e = 0; e < count; e++)
    EXPECT(done[e] == 1, "two-shot count=%zu n=%d G=%d element %zu done %d", count, n, G, e, done[e]);
}

// Reduce-scatter push and all-gather pull: rounds of at most `slot` units,
// every round split as the first (roundRange).
void checkRoundSplit(size_t total, int G, size_t slot, size_t align) {
  const size_t full = total < slot ? total : slot;
  std::vector<unsigned char> done(total, 0);
  std::vector<int> owner(slot, -1);
  for (size_t base = 0; base < total; base += slot) {
    const size_t m = (total - base) < slot ? (total - base) : slot;
    for (int blk = 0; blk < G; blk++) {
      size_t s0, s1;
      roundRange(full, m, G, blk, align, &s0, &s1);
      for (size_t e = s0; e < s1; e++) {
        done[base + e]++;
        EXPECT(owner[e] == -1 || owner[e] == blk, "slot unit %zu used by blocks %d and %d", e, owner[e], blk);
        owner[e] = blk;
      }
    }
  }
  for (size_t e = 0; e < total; e++) EXPECT(done[e] == 1, "round split total=%zu G=%d unit %zu", total, G, e);
}

// Negative control: splitting every round afresh (the chunk recomputed from
// the round's own size) hands some staging bytes to different blocks in
// different rounds; the owner check above must be able to see that.
bool resplitConflicts(size_t total, int n, int G, size_t roundBytes) {
  std::vector<int> owner(roundBytes + 16 * kMaxRanks, -1);
  for (size_t off = 0; off < total; off += roundBytes) {
    const size_t m = (total - off) < roundBytes ? (total - off) : roundBytes;
    const size_t cb = ((m + n - 1) / n + 15) / 16 * 16;
    for (int blk = 0; blk < G; blk++) {
      size_t s0, s1;
      blockRange(cb, G, blk, 16, &s0, &s1);
      for (int q = 0; q < n; q++)
        for (size_t b = q * cb + s0; b < q * cb + s1 && b < m; b++) {
          if (owner[b] != -1 && owner[b] != blk) return true;
          owner[b] = blk;
        }
    }
  }
  return false;
}

// Pipelined NVLS all-reduce (allReduceNvlsPipe): pieces of n chunks rotate
// through kPipeSlots slots; block b owns the same bytes of every slot.
void checkNvlsPipe(size_t total, int n, int G, int pieces, size_t dataBytes) {
  const size_t cb = nvlsPipeChunk(total, n, pieces, dataBytes);
  const size_t slotBytes = nvlsPipeSlotBytes(dataBytes);
  const size_t piece = cb * n;
  EXPECT(cb % 16 == 0 && piece <= slotBytes, "cb %zu slot %zu", cb, slotBytes);
  EXPECT(3 * slotBytes <= dataBytes, "slots exceed the staging region");
  const size_t P = (total + piece - 1) / piece;
  std::vector<unsigned char> in(total, 0), red(total, 0), out(total, 0);
  std::map<size_t, int> owner;  // slot-relative byte -> block
  for (int blk = 0; blk < G; blk++) {
    size_t s0, s1;
    blockRange(cb, G, blk, 16, &s0, &s1);
    for (size_t p = 0; p < P; p++) {
      const size_t off = p * piece, m = (total - off) < piece ? (total - off) : piece;
      for (int q = 0; q < n; q++) {
        const size_t lo = q * cb + s0, hiRaw = q * cb + s1, hi = hiRaw < m ? hiRaw : m;
        for (size_t b = lo; b < hi; b++) {
          in[off + b]++;
          red[off + b]++;
          out[off + b]++;
          auto it = owner.find(b);
          EXPECT(it == owner.end() || it->second == blk, "slot byte %zu used by two blocks", b);
          owner[b] = blk;
          EXPECT((p % 3) * slotBytes + b < 3 * slotBytes, "slot byte out of range");
        }
        if (lo < hi) EXPECT(lo + (hi - lo + 15) / 16 * 16 <= q * cb + s1, "pipe reduce leaves its bytes");
      }
    }
  }
  for (size_t b = 0; b < total; b++)
    EXPECT(in[b] == 1 && red[b] == 1 && out[b] == 1, "pipe total=%zu n=%d G=%d pieces=%d byte %zu", total, n, G,
           pieces, b);
}

// Window all-reduce (allReduceWin + winReduceBroadcast): rank chunks of ce
// elements, block ranges aligned to the pack, packs then an element tail.
void checkWindowAllReduce(size_t count, int n, int G, size_t pk) {
  const size_t ce = rankChunk(count, n, pk);
  std::vector<unsigned char> done(count, 0);
  for (int me = 0; me < n; me++)
    for (int blk = 0; blk < G; blk++) {
      size_t s0, s1;
      blockRange(ce, G, blk, pk, &s0, &s1);
      const size_t lo = me * ce + s0, hiRaw = me * ce + s1, hi = hiRaw < count ? hiRaw : count;
      if (lo >= hi) continue;
      EXPECT(lo % pk == 0, "range start %zu off the pack grid", lo);
      const size_t p0 = lo / pk, p1 = hi / pk;
      for (size_t i = p0; i < p1; i++)
        for (size_t e = i * pk; e < (i + 1) * pk; e++) done[e]++;
      const size_t tail = p1 * pk > lo ? p1 * pk : lo;
      for (size_t e = tail; e < hi; e++) done[e]++;
    }
  for (size_t e = 0; e < count; e++)
    EXPECT(done[e] == 1, "window allreduce count=%zu n=%d G=%d pk=%zu element %zu done %d", count, n, G, pk, e,
           done[e]);
}

// Window reduce-scatter and all-gather: a block split of each rank's part.
void checkWindowScatterGather(size_t rc, int G, size_t pk) {
  std::vector<unsigned char> done(rc, 0);
  for (int blk = 0; blk < G; blk++) {
    size_t s0, s1;
    blockRange(rc, G, blk, pk, &s0, &s1);
    for (size_t e = s0; e < s1; e++) done[e]++;
  }
  for (size_t e = 0; e < rc; e++) EXPECT(done[e] == 1, "window rs/ag rc=%zu G=%d element %zu", rc, G, e);
}

// Split-K fix-up with SiLU*mul: output column j of a tile at col0 takes gate
// column col0 + (jl/16)*32 + jl%16 (jl = j - col0/2), as the reduction kernel
// maps global j to (j/16)*32 + j%16.
void checkFixupSiluMapping() {
  for (int BN : {32, 64, 128, 256})
    for (int tn = 0; tn < 8; tn++) {
      const int col0 = tn * BN;
      std::vector<int> seen(BN / 2, 0);
      for (int idx = 0; idx < BN / 8; idx++) {
        const int jl = 4 * idx;
        const int gcol = col0 + (jl / 16) * 32 + (jl % 16);
        const int j = col0 / 2 + jl;
        EXPECT(gcol == (j / 16) * 32 + (j % 16), "BN=%d tile %d output %d", BN, tn, j);
        EXPECT(gcol + 16 + 3 < col0 + BN, "up columns leave the tile");
        for (int k = 0; k < 4; k++) seen[jl + k]++;
      }
      for (int k = 0; k < BN / 2; k++) EXPECT(seen[k] == 1, "BN=%d output %d covered %d times", BN, k, seen[k]);
    }
}
}  // namespace

int main() {
  const size_t small = 64u << 10;  // staging region sizes that force several rounds
  for (int n : {2, 3, 4, 8})
    for (int G : {1, 3, 8})
      for (size_t total : {size_t(16), size_t(100), size_t(4096 + 48), size_t(70000), size_t(200000)}) {
        checkNvlsRounds(total, n, G, small);
        for (int pieces : {1, 2, 4, 7}) checkNvlsPipe(total, n, G, pieces, small);
      }
  for (int n : {2, 3, 8})
    for (int G : {1, 5, 16})
      for (size_t count : {size_t(1), size_t(999), size_t(5000), size_t(40000)})
        for (size_t pk : {size_t(1), size_t(8)}) checkTwoShot(count, n, G, 2048, pk);
  for (int G : {1, 6, 16})
    for (size_t total : {size_t(10), size_t(4096), size_t(5000), size_t(30001)})
      for (size_t align : {size_t(1), size_t(16)}) checkRoundSplit(total, G, 4096, align);
  for (int n : {2, 5, 8})
    for (int G : {1, 4, 13})
      for (size_t count : {size_t(1), size_t(7), size_t(64), size_t(1000), size_t(4099), size_t(33333)})
        for (size_t pk : {size_t(1), size_t(4), size_t(8), size_t(16)}) {
          checkWindowAllReduce(count, n, G, pk);
          checkWindowScatterGather(count, G, pk);
        }
  checkFixupSiluMapping();
  if (!resplitConflicts(100000, 4, 3, 32768)) {
    std::fprintf(stderr, "FAIL negative control: a per-round re-split showed no conflict\n");
    gFail++;
  }
  if (gFail == 0) std::printf("collective index arithmetic: all checks passed\n");
  return gFail ? 1 : 0;
}
