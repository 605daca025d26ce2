// SPDX-License-Identifier: Apache-2.0
// Out-of-band control plane: unique id, rendezvous, small collectives over
// TCP, and descriptor exchange over Unix sockets.
//
// Capabilities mirror the reference bootstrap (reference:
// src/core/bootstrap.h:19-63, src/core/bootstrap.cc:85-272): the id embeds
// the address of a listening socket bound by vcclGetUniqueId in the rank-0
// process, VCCL_COMM_ID=<ip>:<port> derives the same id on every rank, the
// root validates every joining rank and keeps listening after rejecting a
// stray client, and allGather/barrier run as a star through the root.
//
// Added for the device data plane: every rank reports a host fingerprint
// (all ranks of a device communicator must share one NVLink domain) and
// exchangeFds() hands CUDA VMM / multicast POSIX-fd handles to every peer.
#pragma once

#include <atomic>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "common/net.h"
#include "vccl.h"

namespace vccl {

// Layout of vcclUniqueId.internal.
struct IdLayout {
  uint32_t magic;      // kIdMagic
  uint32_t version;    // VCCL_VERSION_CODE
  uint64_t nonce;      // random per id; kEnvNonce for VCCL_COMM_ID ids
  WireEndpoint root;   // rendezvous address
};
static_assert(sizeof(IdLayout) <= VCCL_UNIQUE_ID_BYTES, "id too large");

constexpr uint32_t kIdMagic = 0x3262766bu;            // "kvb2" little endian
constexpr uint64_t kEnvNonce = 0x454e562d43434c56ull;  // ids from VCCL_COMM_ID

// allowFixed: honour VCCL_COMM_ID (the job's first communicator).  Ids made
// for communicators created later (split) always get a fresh port.
vcclResult_t makeUniqueId(vcclUniqueId* out, bool allowFixed = true);

struct RankInfo {
  uint64_t hostHash;
  int32_t pid;
  int32_t cudaDevice;  // -1 when no device is bound
};

class Bootstrap {
 public:
  static vcclResult_t create(const vcclUniqueId& id, int rank, int nranks,
                             std::unique_ptr<Bootstrap>* out);
  ~Bootstrap();

  int rank() const { return rank_; }
  int nranks() const { return nranks_; }
  uint64_t nonce() const { return nonce_; }

  // Every rank contributes `slice` bytes at buf + rank*slice; on return all
  // ranks hold all slices.
  vcclResult_t allGather(void* buf, size_t slice);
  vcclResult_t barrier();
  // Root's `bytes` at buf are copied to every rank.
  vcclResult_t broadcast(void* buf, size_t bytes, int root);

  // Exchange descriptors: `mine` (same count on every rank) goes to every
  // peer; out[p] receives rank p's descriptors (out[rank] = dup of mine).
  // Caller owns every returned descriptor.
  vcclResult_t exchangeFds(const std::vector<int>& mine,
                           std::vector<std::vector<int>>* out);

  // Rank-to-rank descriptor transfer (used where only one rank exports,
  // e.g. a multicast object created by rank 0).
  vcclResult_t broadcastFds(int root, std::vector<int>* fds, size_t count);

  // Unblock any thread waiting in this bootstrap (vcclCommAbort).
  void abort();

  const std::vector<RankInfo>& ranks() const { return infos_; }
  bool singleHost() const;

 private:
  Bootstrap(int rank, int nranks, uint64_t nonce)
      : rank_(rank), nranks_(nranks), nonce_(nonce) {}
  vcclResult_t rendezvous(const IdLayout& id, int listenFd);
  std::string fdSocketName(int rank, uint64_t seq) const;

  int rank_;
  int nranks_;
  uint64_t nonce_;
  uint64_t fdSeq_ = 0;
  int toRoot_ = -1;              // non-root: connection to the root
  std::vector<int> fromRank_;    // root: connection per rank
  std::vector<RankInfo> infos_;
  std::atomic<bool> aborted_{false};
};

uint64_t hostFingerprint();

// Every rank reports success of a step; all ranks learn whether everyone
// succeeded (so that optional features are enabled or skipped together).
// False on every rank if the exchange itself fails.
bool everyone(Bootstrap* bs, bool mine);

}  // namespace vccl
