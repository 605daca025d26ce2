// SPDX-License-Identifier: Apache-2.0
// Registration cache: the bookkeeping that lets collectives on plain device
// buffers (cudaMalloc memory, PyTorch tensors) run the zero-copy window
// kernels without an explicit vcclCommWindowRegister.
//
// The reference pins every user buffer a call touches and keeps the
// registrations in an LRU cache keyed by address (reference:
// src/core/comm.h:74-139, ScopedReg :185-222, used at
// src/core/collectives.cc:509-511).  On NVLink the costly step is not
// pinning but opening a peer's allocation, and that step is collective: every
// rank must map every peer's buffer.  So a cache entry here is a window that
// every rank registered in the same call, and the cache state that decides
// hits, misses and evictions must stay identical on every rank:
//
// * every entry has an id and a last-use stamp that are the same on every
//   rank (entries are only created, used and dropped by agreed plans);
// * per call each rank reports a fixed-size RegQuery (its own hits, its own
//   stale entries) through one bootstrap allgather, and every rank computes
//   the same RegPlan from the same gathered queries.
//
// A buffer hits an entry when the entry covers it and still belongs to the
// same allocation (the allocation id the driver gives every allocation;
// memory freed and allocated again at the same address has a new id).  The
// call reuses the entry when every rank hits the same entry at the same
// offset (the window kernels address every rank's buffer at one offset).
// Entries of this rank that overlap a buffer without covering it are stale
// and dropped everywhere; so are the entries of a buffer the ranks do not
// hold alike, before it is registered afresh.  Entries of one rank therefore
// never overlap.  This file holds no CUDA calls: the
// window steps are done by the caller (runtime/window.cc), which makes the
// protocol testable on a host without a GPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace vccl {

constexpr int kRegMaxBuffers = 2;  // send and receive
constexpr int kRegMaxStale = 4;
constexpr int32_t kRegNone = -1;        // no entry holds the buffer
constexpr int32_t kRegUserWindow = -2;  // an explicitly registered window holds it

// One buffer of a call as this rank sees it.
struct RegKey {
  uintptr_t ptr = 0;
  size_t bytes = 0;
  uint64_t allocId = 0;    // the allocation's id (0 if unknown: never cached)
  bool userWindow = false;  // lies in an explicitly registered window
};

// One rank's report for one call (travels through the bootstrap allgather,
// so it is plain data of fixed size).
struct RegQuery {
  int32_t eligible = 0;  // every buffer can be cached on this rank
  int32_t nbuf = 0;
  int32_t hit[kRegMaxBuffers] = {kRegNone, kRegNone};
  uint64_t off[kRegMaxBuffers] = {0, 0};  // the buffer's offset inside its hit entry
  int32_t stale[kRegMaxStale] = {kRegNone, kRegNone, kRegNone, kRegNone};
  int32_t staleOverflow = 0;  // more stale entries than fit: drop everything
  int32_t pad = 0;
};

// What every rank does for the call, identical on every rank.
struct RegPlan {
  bool take = false;                  // the call runs on cached windows
  std::vector<int32_t> evict;         // entries every rank drops first (ascending)
  bool reg[kRegMaxBuffers] = {false, false};  // buffer i gets a new entry on every rank
  int32_t use[kRegMaxBuffers] = {kRegNone, kRegNone};  // entry of buffer i when reused
};

struct RegEntry {
  int32_t id = kRegNone;
  uint64_t lastUse = 0;
  uintptr_t ptr = 0;
  size_t bytes = 0;
  uint64_t allocId = 0;
  void* handle = nullptr;  // the window (owned by the caller)
};

struct RegStats {
  uint64_t calls = 0;      // calls that consulted the cache with every rank eligible
  uint64_t hits = 0;       // buffers served by an existing entry
  uint64_t misses = 0;     // buffers that were registered
  uint64_t evictions = 0;  // entries dropped (stale, capacity or flush)
};

// Entries the cache may hold: VCCL_REG_CACHE_ENTRIES, else the reference's
// VCCL_MR_CACHE, else 16 (at least kRegMaxBuffers).
int regCacheCapacityFromEnv();

class RegCacheBook {
 public:
  explicit RegCacheBook(int capacity = 32) : capacity_(capacity < kRegMaxBuffers ? kRegMaxBuffers : capacity) {}

  int capacity() const { return capacity_; }
  void setCapacity(int c) { capacity_ = c < kRegMaxBuffers ? kRegMaxBuffers : c; }
  void* handleOf(int32_t id) const {
    const RegEntry* e = find(id);
    return e ? e->handle : nullptr;
  }
  const std::vector<RegEntry>& entries() const { return entries_; }
  const RegStats& stats() const { return stats_; }

  // This rank's report.  `eligible` is false when some buffer cannot be
  // cached here (not plain device memory, no allocation id, the stream is
  // being captured, buffers overlap); the query then only says so.
  RegQuery query(const RegKey* keys, int nbuf, bool eligible) const;

  // The call's plan from every rank's query ([rank] order).  Pure: every
  // rank that holds the same book and sees the same queries gets the same
  // plan.
  RegPlan plan(const std::vector<RegQuery>& all) const;

  // Bookkeeping after the plan's window steps (same order on every rank):
  // drop an entry, add a new one (returns its id), mark an entry used.
  void* drop(int32_t id);
  int32_t add(const RegKey& key, void* handle);
  void touch(int32_t id);
  // Ids of every entry, ascending (a flush drops them all).
  std::vector<int32_t> ids() const;

  void countCall(const RegPlan& p);

 private:
  const RegEntry* find(int32_t id) const;

  int capacity_;
  int32_t nextId_ = 0;
  uint64_t clock_ = 0;
  std::vector<RegEntry> entries_;
  RegStats stats_;
};

}  // namespace vccl
