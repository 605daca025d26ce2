// SPDX-License-Identifier: Apache-2.0
// Registration-cache bookkeeping (host only; see regcache.h).
#include "runtime/regcache.h"

#include <algorithm>

#include "common/env.h"

namespace vccl {

int regCacheCapacityFromEnv() {
  const long cap = envLong("VCCL_REG_CACHE_ENTRIES", envLong("VCCL_MR_CACHE", 16));
  return cap < kRegMaxBuffers ? kRegMaxBuffers : cap > (1 << 20) ? (1 << 20) : static_cast<int>(cap);
}

RegQuery RegCacheBook::query(const RegKey* keys, int nbuf, bool eligible) const {
  RegQuery q;
  q.nbuf = nbuf;
  q.eligible = eligible && nbuf >= 1 && nbuf <= kRegMaxBuffers ? 1 : 0;
  if (!q.eligible) return q;
  int nstale = 0;
  for (int i = 0; i < nbuf; i++) {
    const RegKey& k = keys[i];
    if (k.userWindow) {
      q.hit[i] = kRegUserWindow;
      continue;
    }
    if (k.allocId == 0 || k.bytes == 0) {
      q.eligible = 0;
      return q;
    }
    for (const RegEntry& e : entries_) {
      const bool overlaps = e.ptr < k.ptr + k.bytes && k.ptr < e.ptr + e.bytes;
      if (!overlaps) continue;
      if (e.ptr <= k.ptr && k.ptr + k.bytes <= e.ptr + e.bytes && e.allocId == k.allocId &&
          q.hit[i] == kRegNone) {
        q.hit[i] = e.id;
        q.off[i] = static_cast<uint64_t>(k.ptr - e.ptr);
        continue;
      }
      // Overlapping without covering: the allocation was replaced, or the
      // buffer runs past a cached range.
      bool seen = false;
      for (int s = 0; s < nstale; s++) seen |= q.stale[s] == e.id;
      if (seen) continue;
      if (nstale == kRegMaxStale) {
        q.staleOverflow = 1;
      } else {
        q.stale[nstale++] = e.id;
      }
    }
  }
  return q;
}

RegPlan RegCacheBook::plan(const std::vector<RegQuery>& all) const {
  RegPlan p;
  if (all.empty()) return p;
  const int nbuf = all[0].nbuf;
  for (const RegQuery& q : all)
    if (!q.eligible || q.nbuf != nbuf) return p;
  // A buffer in an explicit window on any rank: the window rule governs the
  // call (it runs on the user's windows when every rank has them).
  for (const RegQuery& q : all)
    for (int i = 0; i < nbuf; i++)
      if (q.hit[i] == kRegUserWindow) return p;
  p.take = true;

  std::vector<int32_t> evict;
  bool flushAll = false;
  for (const RegQuery& q : all) {
    flushAll |= q.staleOverflow != 0;
    for (int s = 0; s < kRegMaxStale; s++)
      if (q.stale[s] != kRegNone) evict.push_back(q.stale[s]);
  }
  if (flushAll) {
    evict = ids();
  }
  auto evicted = [&](int32_t id) { return std::find(evict.begin(), evict.end(), id) != evict.end(); };
  // A buffer not held alike everywhere drops every rank's entry for it, which
  // can take away the entry another buffer of the call was going to reuse:
  // repeat until nothing changes (a buffer only ever moves to "register").
  for (bool changed = true; changed;) {
    changed = false;
    for (int i = 0; i < nbuf; i++) {
      if (p.reg[i]) continue;
      const int32_t first = all[0].hit[i];
      bool same = first >= 0 && !evicted(first);
      for (const RegQuery& q : all) same &= q.hit[i] == first && q.off[i] == all[0].off[i];
      if (same) {
        p.use[i] = first;
        continue;
      }
      p.use[i] = kRegNone;
      p.reg[i] = true;
      changed = true;
      for (const RegQuery& q : all)
        if (q.hit[i] >= 0 && !evicted(q.hit[i])) evict.push_back(q.hit[i]);
    }
  }
  // Room for the new entries: least recently used first, never an entry
  // this call reuses.
  std::sort(evict.begin(), evict.end());
  evict.erase(std::unique(evict.begin(), evict.end()), evict.end());
  // Ids that some rank reported but that are not in this book cannot occur
  // while the books agree; keep only known ones so every rank drops the same.
  evict.erase(std::remove_if(evict.begin(), evict.end(), [&](int32_t id) { return find(id) == nullptr; }),
              evict.end());
  int fresh = 0;
  for (int i = 0; i < nbuf; i++) fresh += p.reg[i] ? 1 : 0;
  long count = static_cast<long>(entries_.size()) - static_cast<long>(evict.size()) + fresh;
  if (count > capacity_) {
    std::vector<const RegEntry*> lru;
    for (const RegEntry& e : entries_) {
      if (evicted(e.id)) continue;
      bool used = false;
      for (int i = 0; i < nbuf; i++) used |= p.use[i] == e.id;
      if (!used) lru.push_back(&e);
    }
    std::sort(lru.begin(), lru.end(), [](const RegEntry* a, const RegEntry* b) {
      return a->lastUse != b->lastUse ? a->lastUse < b->lastUse : a->id < b->id;
    });
    for (const RegEntry* e : lru) {
      if (count <= capacity_) break;
      evict.push_back(e->id);
      count--;
    }
    std::sort(evict.begin(), evict.end());
  }
  p.evict = evict;
  return p;
}

const RegEntry* RegCacheBook::find(int32_t id) const {
  for (const RegEntry& e : entries_)
    if (e.id == id) return &e;
  return nullptr;
}

void* RegCacheBook::drop(int32_t id) {
  for (size_t i = 0; i < entries_.size(); i++) {
    if (entries_[i].id == id) {
      void* h = entries_[i].handle;
      entries_.erase(entries_.begin() + static_cast<long>(i));
      stats_.evictions++;
      return h;
    }
  }
  return nullptr;
}

int32_t RegCacheBook::add(const RegKey& key, void* handle) {
  RegEntry e;
  e.id = nextId_++;
  e.lastUse = ++clock_;
  e.ptr = key.ptr;
  e.bytes = key.bytes;
  e.allocId = key.allocId;
  e.handle = handle;
  entries_.push_back(e);
  stats_.misses++;
  return e.id;
}

void RegCacheBook::touch(int32_t id) {
  for (RegEntry& e : entries_) {
    if (e.id == id) {
      e.lastUse = ++clock_;
      stats_.hits++;
      return;
    }
  }
}

std::vector<int32_t> RegCacheBook::ids() const {
  std::vector<int32_t> v;
  for (const RegEntry& e : entries_) v.push_back(e.id);
  std::sort(v.begin(), v.end());
  return v;
}

void RegCacheBook::countCall(const RegPlan& p) {
  if (p.take) stats_.calls++;
}

}  // namespace vccl
