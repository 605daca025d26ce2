// SPDX-License-Identifier: Apache-2.0
// Registration-cache protocol on the host: several simulated ranks, each
// with its own RegCacheBook and its own address layout, run random call
// sequences (buffers reused, freed and allocated again at the same or
// another address, a rank now and then unable to take part, application
// windows).  After every call the checks are:
//   * every rank computed the same plan, and the books agree on every
//     entry's id and last use;
//   * a call that runs on cached windows has, for every buffer, a window on
//     every rank that covers the buffer, at one offset on every rank, over
//     the buffer's current allocation;
//   * entries of one rank never overlap, and never exceed the capacity.
// A negative control checks that the offset agreement is what keeps a call
// off the cache when the ranks' buffers sit at different offsets.
#include <algorithm>
#include <array>
#include <cstdint>
#include <cstdio>
#include <map>
#include <vector>

#include "runtime/regcache.h"

using namespace vccl;

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

struct Rng {
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed * 2654435761u + 1) {}
  uint32_t next() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return static_cast<uint32_t>(s >> 11);
  }
  uint32_t below(uint32_t n) { return next() % n; }
};

// A simulated window: the range it was registered over on its rank.
struct FakeWindow {
  uintptr_t ptr;
  size_t bytes;
  uint64_t allocId;
};

// One rank's memory: logical tensor t lives at base[t] in allocation id[t].
struct RankMem {
  std::vector<uintptr_t> base;
  std::vector<uint64_t> id;
};

constexpr int kTensors = 12;
constexpr size_t kTensorBytes = 64u << 20;

struct Sim {
  int nranks;
  int capacity;
  std::vector<RegCacheBook> books;
  std::vector<RankMem> mem;
  std::vector<std::map<int32_t, FakeWindow*>> windows;  // per rank: entry id -> window
  uint64_t nextId = 1;
  uintptr_t nextAddr = 0x7f0000000000ull;
  uint64_t takes = 0, hits = 0, regs = 0;

  Sim(int n, int cap, Rng& rng) : nranks(n), capacity(cap), books(n, RegCacheBook(cap)), mem(n), windows(n) {
    for (int r = 0; r < n; r++) {
      for (int t = 0; t < kTensors; t++) {
        // Different layouts per rank: the same logical tensor has another
        // address on every rank.
        mem[r].base.push_back(nextAddr + (static_cast<uintptr_t>(rng.below(32)) << 21));  // tensors never overlap
        nextAddr += 2 * kTensorBytes + (static_cast<uintptr_t>(rng.below(8)) << 21);
        mem[r].id.push_back(nextId++);
      }
    }
  }
  ~Sim() {
    for (auto& m : windows)
      for (auto& kv : m) delete kv.second;
  }

  // Rank r frees tensor t and gets it back at the same address (new id) or
  // at a new one.
  void realloc(int r, int t, bool sameAddress) {
    mem[r].id[t] = nextId++;
    if (!sameAddress) {
      mem[r].base[t] = nextAddr;
      nextAddr += 2 * kTensorBytes;
    }
  }

  // One call on buffers (tensor, offset, bytes); offsets may differ per rank.
  // Returns whether the call ran on cached windows.
  bool call(const std::vector<std::vector<std::array<uint64_t, 3>>>& perRank, const std::vector<bool>& eligible,
            const std::vector<bool>& userWin, const char* tag) {
    const int nbuf = static_cast<int>(perRank[0].size());
    std::vector<RegQuery> all(nranks);
    std::vector<std::vector<RegKey>> keys(nranks);
    for (int r = 0; r < nranks; r++) {
      for (int i = 0; i < nbuf; i++) {
        RegKey k;
        const int t = static_cast<int>(perRank[r][i][0]);
        k.ptr = mem[r].base[t] + perRank[r][i][1];
        k.bytes = perRank[r][i][2];
        k.allocId = mem[r].id[t];
        k.userWindow = userWin[r];
        keys[r].push_back(k);
      }
      all[r] = books[r].query(keys[r].data(), nbuf, eligible[r]);
    }
    std::vector<RegPlan> plans;
    for (int r = 0; r < nranks; r++) plans.push_back(books[r].plan(all));
    for (int r = 1; r < nranks; r++) {
      EXPECT(plans[r].take == plans[0].take && plans[r].evict == plans[0].evict &&
                 plans[r].reg[0] == plans[0].reg[0] && plans[r].reg[1] == plans[0].reg[1] &&
                 plans[r].use[0] == plans[0].use[0] && plans[r].use[1] == plans[0].use[1],
             "%s: rank %d planned differently from rank 0", tag, r);
    }
    const RegPlan& p = plans[0];
    if (!p.take) return false;
    takes++;
    std::vector<std::vector<FakeWindow*>> got(nranks, std::vector<FakeWindow*>(nbuf, nullptr));
    for (int r = 0; r < nranks; r++) {
      RegCacheBook& b = books[r];
      for (int32_t id : p.evict) {
        FakeWindow* w = static_cast<FakeWindow*>(b.drop(id));
        EXPECT(w != nullptr, "%s: rank %d evicts unknown entry %d", tag, r, id);
        windows[r].erase(id);
        delete w;
      }
      for (int i = 0; i < nbuf; i++) {
        if (p.use[i] >= 0) {
          b.touch(p.use[i]);
          got[r][i] = static_cast<FakeWindow*>(b.handleOf(p.use[i]));
          if (r == 0) hits++;
        } else if (p.reg[i]) {
          auto* w = new FakeWindow{keys[r][i].ptr, keys[r][i].bytes, keys[r][i].allocId};
          const int32_t id = b.add(keys[r][i], w);
          windows[r][id] = w;
          got[r][i] = w;
          if (r == 0) regs++;
        }
      }
    }
    // Every buffer covered on every rank, at one offset, by its current allocation.
    for (int i = 0; i < nbuf; i++) {
      uint64_t off0 = 0;
      for (int r = 0; r < nranks; r++) {
        FakeWindow* w = got[r][i];
        EXPECT(w != nullptr, "%s: buffer %d has no window on rank %d", tag, i, r);
        if (w == nullptr) continue;
        const RegKey& k = keys[r][i];
        EXPECT(w->ptr <= k.ptr && k.ptr + k.bytes <= w->ptr + w->bytes, "%s: window misses buffer %d on rank %d",
               tag, i, r);
        EXPECT(w->allocId == k.allocId, "%s: rank %d buffer %d served by a replaced allocation", tag, r, i);
        const uint64_t off = k.ptr - w->ptr;
        if (r == 0) off0 = off;
        EXPECT(off == off0, "%s: buffer %d at offset %llu on rank %d, %llu on rank 0", tag, i,
               static_cast<unsigned long long>(off), r, static_cast<unsigned long long>(off0));
      }
    }
    checkBooks(tag);
    return true;
  }

  void checkBooks(const char* tag) {
    const auto& e0 = books[0].entries();
    for (int r = 0; r < nranks; r++) {
      const auto& e = books[r].entries();
      EXPECT(static_cast<int>(e.size()) <= capacity, "%s: rank %d holds %zu entries (capacity %d)", tag, r, e.size(),
             capacity);
      EXPECT(e.size() == e0.size(), "%s: rank %d holds %zu entries, rank 0 %zu", tag, r, e.size(), e0.size());
      for (size_t a = 0; a < e.size() && a < e0.size(); a++)
        EXPECT(e[a].id == e0[a].id && e[a].lastUse == e0[a].lastUse, "%s: rank %d entry %zu differs", tag, r, a);
      for (size_t a = 0; a < e.size(); a++)
        for (size_t b2 = a + 1; b2 < e.size(); b2++)
          EXPECT(!(e[a].ptr < e[b2].ptr + e[b2].bytes && e[b2].ptr < e[a].ptr + e[a].bytes),
                 "%s: rank %d entries %d and %d overlap", tag, r, e[a].id, e[b2].id);
    }
  }
};

using Buf = std::array<uint64_t, 3>;

void randomRun(uint64_t seed, int nranks, int cap, int calls) {
  Rng rng(seed);
  Sim sim(nranks, cap, rng);
  char tag[64];
  for (int c = 0; c < calls; c++) {
    std::snprintf(tag, sizeof(tag), "seed %llu call %d", static_cast<unsigned long long>(seed), c);
    const uint32_t ev = rng.below(100);
    if (ev < 8) {
      sim.realloc(static_cast<int>(rng.below(nranks)), static_cast<int>(rng.below(kTensors)), rng.below(2) == 0);
      continue;
    }
    const int nbuf = 1 + static_cast<int>(rng.below(2));
    int t0 = static_cast<int>(rng.below(kTensors));
    int t1 = (t0 + 1 + static_cast<int>(rng.below(kTensors - 1))) % kTensors;
    // Sizes and offsets agree across ranks (the collective's contract);
    // offsets are sub-ranges of a tensor now and then (slices).
    const uint64_t bytes = (rng.below(4) == 0 ? 16u : 64u) << 20;
    const uint64_t off0 = bytes == kTensorBytes ? 0 : (static_cast<uint64_t>(rng.below(3)) << 24);
    const uint64_t off1 = bytes == kTensorBytes ? 0 : (static_cast<uint64_t>(rng.below(3)) << 24);
    // Now and then every rank slices its tensor at its own offset (pointers
    // are per rank; only sizes must agree).
    const bool skew = bytes != kTensorBytes && rng.below(10) == 0;
    std::vector<std::vector<Buf>> per(nranks);
    for (int r = 0; r < nranks; r++) {
      const uint64_t o0 = skew ? (static_cast<uint64_t>(rng.below(3)) << 24) : off0;
      per[r].push_back({static_cast<uint64_t>(t0), o0, bytes});
      if (nbuf == 2) per[r].push_back({static_cast<uint64_t>(t1), off1, bytes});
    }
    std::vector<bool> eligible(nranks, true), user(nranks, false);
    if (rng.below(20) == 0) eligible[rng.below(nranks)] = false;  // a rank captures or staged a host buffer
    if (rng.below(25) == 0) std::fill(user.begin(), user.end(), true);
    sim.call(per, eligible, user, tag);
  }
  EXPECT(sim.takes > 0 && sim.hits > 0 && sim.regs > 0, "seed %llu: takes %llu hits %llu regs %llu",
         static_cast<unsigned long long>(seed), static_cast<unsigned long long>(sim.takes),
         static_cast<unsigned long long>(sim.hits), static_cast<unsigned long long>(sim.regs));
}

void directedCases() {
  Rng rng(7);
  Sim sim(4, 4, rng);
  std::vector<bool> yes(4, true), no(4, false);
  auto one = [&](int t, uint64_t off, uint64_t bytes) {
    return std::vector<std::vector<Buf>>(4, std::vector<Buf>{{static_cast<uint64_t>(t), off, bytes}});
  };
  // First call registers, the second reuses.
  EXPECT(sim.call(one(0, 0, kTensorBytes), yes, no, "first"), "first call not cached");
  EXPECT(sim.regs == 1 && sim.hits == 0, "first call: regs %llu hits %llu", (unsigned long long)sim.regs,
         (unsigned long long)sim.hits);
  EXPECT(sim.call(one(0, 0, kTensorBytes), yes, no, "second"), "second call not cached");
  EXPECT(sim.regs == 1 && sim.hits == 1, "second call: regs %llu hits %llu", (unsigned long long)sim.regs,
         (unsigned long long)sim.hits);
  // A slice at one offset on every rank reuses the entry.
  EXPECT(sim.call(one(0, 16u << 20, 16u << 20), yes, no, "slice"), "slice not cached");
  EXPECT(sim.regs == 1 && sim.hits == 2, "slice: regs %llu hits %llu", (unsigned long long)sim.regs,
         (unsigned long long)sim.hits);
  // Rank 2 frees the tensor and gets the same address back: a new
  // registration, never the old window.
  sim.realloc(2, 0, true);
  EXPECT(sim.call(one(0, 0, kTensorBytes), yes, no, "realloc"), "realloc call not cached");
  EXPECT(sim.regs == 2, "realloc: regs %llu", (unsigned long long)sim.regs);
  EXPECT(sim.books[0].stats().evictions == 1, "realloc: evictions %llu",
         (unsigned long long)sim.books[0].stats().evictions);
  // One rank unable to take part keeps every rank off the cache.
  std::vector<bool> oneOut(4, true);
  oneOut[3] = false;
  EXPECT(!sim.call(one(0, 0, kTensorBytes), oneOut, no, "ineligible"), "ineligible rank still cached");
  // Application windows take precedence.
  EXPECT(!sim.call(one(0, 0, kTensorBytes), yes, yes, "user"), "user window call went to the cache");
  // Capacity: five tensors through a 4-entry cache drop the least recently used.
  for (int t = 1; t <= 4; t++) sim.call(one(t, 0, kTensorBytes), yes, no, "fill");
  EXPECT(sim.books[0].entries().size() == 4, "capacity: %zu entries", sim.books[0].entries().size());
  const uint64_t before = sim.regs;
  sim.call(one(1, 0, kTensorBytes), yes, no, "lru-hit");  // tensor 1 is still cached
  EXPECT(sim.regs == before, "tensor 1 was evicted too early");
  sim.call(one(0, 0, kTensorBytes), yes, no, "lru-miss");  // tensor 0 was the oldest
  EXPECT(sim.regs == before + 1, "tensor 0 should have been re-registered");

  // Negative control: offsets that differ across ranks must not reuse an
  // entry (the window kernels address every rank at one offset).
  std::vector<std::vector<Buf>> skew(4);
  for (int r = 0; r < 4; r++) skew[r].push_back({1, r == 1 ? (16u << 20) : 0, 16u << 20});
  const uint64_t hitsBefore = sim.hits, regsBefore = sim.regs;
  EXPECT(sim.call(skew, yes, no, "skew"), "skewed call not cached at all");
  EXPECT(sim.hits == hitsBefore && sim.regs == regsBefore + 1,
         "skewed offsets reused an entry (hits %llu -> %llu)", (unsigned long long)hitsBefore,
         (unsigned long long)sim.hits);
}

// The reference's cache scenario (capacity 4; reference:
// tests/test_mrcache.cc): seven distinct buffers in seven calls register
// seven times and drop three; the four newest stay.
// Reusing the oldest survivor makes the next registration drop the one after
// it instead.  A flush then drops everything.
void lruScenario() {
  Rng rng(11);
  Sim sim(2, 4, rng);
  std::vector<bool> yes(2, true), no(2, false);
  auto one = [&](int t) {
    return std::vector<std::vector<Buf>>(2, std::vector<Buf>{{static_cast<uint64_t>(t), 0, kTensorBytes}});
  };
  auto cached = [&](int t) {
    for (const RegEntry& e : sim.books[0].entries())
      if (e.ptr == sim.mem[0].base[t]) return true;
    return false;
  };
  for (int t = 0; t < 7; t++) sim.call(one(t), yes, no, "lru fill");
  EXPECT(sim.regs == 7 && sim.books[0].stats().evictions == 3 && sim.books[0].entries().size() == 4,
         "lru: regs %llu evictions %llu entries %zu", (unsigned long long)sim.regs,
         (unsigned long long)sim.books[0].stats().evictions, sim.books[0].entries().size());
  for (int t = 0; t < 3; t++) EXPECT(!cached(t), "lru: buffer %d should have been dropped", t);
  for (int t = 3; t < 7; t++) EXPECT(cached(t), "lru: buffer %d should be cached", t);
  sim.call(one(3), yes, no, "lru touch");  // reuse the oldest survivor
  EXPECT(sim.hits == 1, "lru: buffer 3 was not reused");
  sim.call(one(7), yes, no, "lru eighth");
  EXPECT(cached(3) && !cached(4), "lru: the reused buffer must survive and buffer 4 go");
  EXPECT(sim.books[0].entries().size() == 4, "lru: %zu entries", sim.books[0].entries().size());
  // Flush: every rank drops every entry, in the same order.
  const std::vector<int32_t> ids0 = sim.books[0].ids();
  for (int r = 0; r < 2; r++) {
    EXPECT(sim.books[r].ids() == ids0, "flush: rank %d holds other ids", r);
    for (int32_t id : sim.books[r].ids()) {
      delete static_cast<FakeWindow*>(sim.books[r].drop(id));
      sim.windows[r].erase(id);
    }
    EXPECT(sim.books[r].entries().empty(), "flush: rank %d not empty", r);
  }
}

}  // namespace

int main() {
  directedCases();
  lruScenario();
  int runs = 0;
  for (int nranks : {2, 3, 8})
    for (int cap : {2, 4, 32})
      for (uint64_t seed = 1; seed <= 6; seed++, runs++) randomRun(seed * 131 + nranks * 7 + cap, nranks, cap, 400);
  if (gFail) {
    std::printf("regcache: %d failures\n", gFail);
    return 1;
  }
  std::printf("regcache: OK (%d random runs)\n", runs);
  return 0;
}
