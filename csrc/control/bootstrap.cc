// SPDX-License-Identifier: Apache-2.0
// Unique id, rendezvous through the root, allGather / barrier / broadcast and
// descriptor exchange (reference: src/core/bootstrap.cc:85-272).
#include "control/bootstrap.h"

#include <arpa/inet.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <random>

#include "common/env.h"
#include "common/log.h"

namespace vccl {
namespace {

// Listening sockets bound by makeUniqueId, keyed by nonce, until the rank-0
// communicator of that id claims them.
std::mutex gListenMu;
std::map<uint64_t, int> gListenByNonce;

constexpr uint32_t kOrderTag = 0x01020304u;

struct JoinRecord {
  uint32_t magic;
  uint32_t version;
  uint64_t nonce;
  int32_t nranks;
  int32_t rank;
  uint32_t orderTag;  // written natively: a peer of other byte order reads it swapped
  int32_t reserved;
  RankInfo info;
};
static_assert(sizeof(JoinRecord) == 48, "join record layout");

uint64_t fnv1a(const void* p, size_t n, uint64_t h = 1469598103934665603ull) {
  const unsigned char* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 1099511628211ull;
  return h;
}

}  // namespace

uint64_t hostFingerprint() {
  char name[256] = {0};
  gethostname(name, sizeof(name) - 1);
  uint64_t h = fnv1a(name, strlen(name));
  std::ifstream boot("/proc/sys/kernel/random/boot_id");
  std::string id;
  if (boot && std::getline(boot, id)) h = fnv1a(id.data(), id.size(), h);
  return h;
}

vcclResult_t makeUniqueId(vcclUniqueId* out, bool allowFixed) {
  memset(out->internal, 0, sizeof(out->internal));
  IdLayout id{};
  id.magic = kIdMagic;
  id.version = VCCL_VERSION_CODE;

  std::string fixed = allowFixed ? envStr("VCCL_COMM_ID", "") : std::string();
  if (!fixed.empty()) {
    // Every rank computes the same id; rank 0 binds the port when it joins.
    if (parseEndpoint(fixed.c_str(), &id.root) != vcclSuccess) {
      VERR("VCCL_COMM_ID must be <ip>:<port>, got '%s'", fixed.c_str());
      return vcclInvalidArgument;
    }
    id.nonce = kEnvNonce;
    memcpy(out->internal, &id, sizeof(id));
    VINFO("unique id from VCCL_COMM_ID=%s", fixed.c_str());
    return vcclSuccess;
  }

  VTRY(localEndpoint(&id.root));
  int lfd = -1;
  uint16_t port = 0;
  VTRY(tcpListen(0, &lfd, &port));
  id.root.portBE = htons(port);
  std::random_device rd;
  do {
    id.nonce = (static_cast<uint64_t>(rd()) << 32) ^ rd() ^
               (static_cast<uint64_t>(getpid()) << 17);
  } while (id.nonce == kEnvNonce || id.nonce == 0);
  {
    std::lock_guard<std::mutex> g(gListenMu);
    gListenByNonce[id.nonce] = lfd;
  }
  memcpy(out->internal, &id, sizeof(id));
  VINFO("unique id created; root listens at %s", endpointString(id.root).c_str());
  return vcclSuccess;
}

vcclResult_t Bootstrap::create(const vcclUniqueId& uid, int rank, int nranks,
                               std::unique_ptr<Bootstrap>* out) {
  IdLayout id;
  memcpy(&id, uid.internal, sizeof(id));
  if (id.magic != kIdMagic) {
    VERR("invalid unique id (bad magic)");
    return vcclInvalidArgument;
  }
  std::unique_ptr<Bootstrap> bs(new Bootstrap(rank, nranks, id.nonce));
  int lfd = -1;
  if (rank == 0) {
    {
      std::lock_guard<std::mutex> g(gListenMu);
      auto it = gListenByNonce.find(id.nonce);
      if (it != gListenByNonce.end()) {
        lfd = it->second;
        gListenByNonce.erase(it);
      }
    }
    if (lfd < 0 && id.nonce == kEnvNonce) VTRY(tcpListen(endpointPort(id.root), &lfd, nullptr));
    if (lfd < 0 && nranks > 1) {
      VERR("rank 0 must join from the process that created the unique id "
           "(or set VCCL_COMM_ID)");
      return vcclInvalidUsage;
    }
  }
  vcclResult_t res = bs->rendezvous(id, lfd);
  closeFd(lfd);
  if (res != vcclSuccess) return res;
  *out = std::move(bs);
  return vcclSuccess;
}

vcclResult_t Bootstrap::rendezvous(const IdLayout& id, int listenFd) {
  RankInfo me{hostFingerprint(), static_cast<int32_t>(getpid()), -1};
  infos_.assign(nranks_, RankInfo{});
  infos_[rank_] = me;
  if (nranks_ == 1) return vcclSuccess;

  if (rank_ != 0) {
    VTRY(tcpConnect(id.root, connectWindowMs(), &toRoot_));
    JoinRecord jr{};
    jr.magic = id.magic;
    jr.version = VCCL_VERSION_CODE;
    jr.nonce = id.nonce;
    jr.nranks = nranks_;
    jr.rank = rank_;
    jr.orderTag = kOrderTag;
    jr.info = me;
    VTRY(sendFull(toRoot_, &jr, sizeof(jr), &aborted_));
    uint8_t verdict = 0;
    VTRY(recvFull(toRoot_, &verdict, 1, &aborted_));
    if (verdict != 1) {
      VERR("bootstrap: root rejected rank %d (id/version/size/rank mismatch)", rank_);
      return vcclInvalidUsage;
    }
    VTRY(recvFull(toRoot_, infos_.data(), sizeof(RankInfo) * nranks_, &aborted_));
    return vcclSuccess;
  }

  fromRank_.assign(nranks_, -1);
  int joined = 0;
  while (joined < nranks_ - 1) {
    int cfd = -1;
    VTRY(tcpAccept(listenFd, &aborted_, &cfd));
    JoinRecord jr{};
    vcclResult_t rr = recvFull(cfd, &jr, sizeof(jr), &aborted_);
    bool good = rr == vcclSuccess && jr.magic == id.magic && jr.nonce == id.nonce &&
                jr.version == static_cast<uint32_t>(VCCL_VERSION_CODE) &&
                jr.orderTag == kOrderTag && jr.nranks == nranks_ && jr.rank > 0 &&
                jr.rank < nranks_ && fromRank_[jr.rank] < 0;
    uint8_t verdict = good ? 1 : 0;
    (void)sendFull(cfd, &verdict, 1);
    if (!good) {
      // One bad client must not break a job that is still forming.
      VWARN("bootstrap: rejected a joining client; %d rank(s) still expected",
            nranks_ - 1 - joined);
      closeFd(cfd);
      continue;
    }
    fromRank_[jr.rank] = cfd;
    infos_[jr.rank] = jr.info;
    joined++;
  }
  for (int r = 1; r < nranks_; r++)
    VTRY(sendFull(fromRank_[r], infos_.data(), sizeof(RankInfo) * nranks_, &aborted_));
  return vcclSuccess;
}

Bootstrap::~Bootstrap() {
  closeFd(toRoot_);
  for (int fd : fromRank_) closeFd(fd);
}

void Bootstrap::abort() {
  aborted_.store(true);
  shutdownFd(toRoot_);
  for (int fd : fromRank_) shutdownFd(fd);
}

bool Bootstrap::singleHost() const {
  for (const RankInfo& r : infos_)
    if (r.hostHash != infos_[0].hostHash) return false;
  return true;
}

vcclResult_t Bootstrap::allGather(void* buf, size_t slice) {
  if (nranks_ == 1 || slice == 0) return vcclSuccess;
  char* b = static_cast<char*>(buf);
  if (rank_ == 0) {
    for (int r = 1; r < nranks_; r++)
      VTRY(recvFull(fromRank_[r], b + r * slice, slice, &aborted_));
    for (int r = 1; r < nranks_; r++)
      VTRY(sendFull(fromRank_[r], b, slice * nranks_, &aborted_));
    return vcclSuccess;
  }
  VTRY(sendFull(toRoot_, b + rank_ * slice, slice, &aborted_));
  return recvFull(toRoot_, b, slice * nranks_, &aborted_);
}

bool everyone(Bootstrap* bs, bool mine) {
  std::vector<uint8_t> v(bs->nranks(), 0);
  v[bs->rank()] = mine ? 1 : 0;
  if (bs->allGather(v.data(), 1) != vcclSuccess) return false;
  for (uint8_t x : v)
    if (!x) return false;
  return true;
}

vcclResult_t Bootstrap::barrier() {
  std::vector<uint8_t> tok(nranks_, 1);
  return allGather(tok.data(), 1);
}

vcclResult_t Bootstrap::broadcast(void* buf, size_t bytes, int root) {
  if (nranks_ == 1 || bytes == 0) return vcclSuccess;
  // Root -> rank 0 (if needed), then rank 0 -> everyone.
  char* b = static_cast<char*>(buf);
  if (root != 0) {
    if (rank_ == root) VTRY(sendFull(toRoot_, b, bytes, &aborted_));
    if (rank_ == 0) VTRY(recvFull(fromRank_[root], b, bytes, &aborted_));
  }
  if (rank_ == 0) {
    for (int r = 1; r < nranks_; r++)
      VTRY(sendFull(fromRank_[r], b, bytes, &aborted_));
    return vcclSuccess;
  }
  return recvFull(toRoot_, b, bytes, &aborted_);
}

std::string Bootstrap::fdSocketName(int rank, uint64_t seq) const {
  char name[96];
  std::snprintf(name, sizeof(name), "vccl-b200-%016llx-%llu-%d",
                static_cast<unsigned long long>(nonce_),
                static_cast<unsigned long long>(seq), rank);
  return name;
}

vcclResult_t Bootstrap::exchangeFds(const std::vector<int>& mine,
                                    std::vector<std::vector<int>>* out) {
  out->assign(nranks_, {});
  for (int fd : mine) (*out)[rank_].push_back(dup(fd));
  if (nranks_ == 1) return vcclSuccess;
  if (!singleHost()) {
    VERR("descriptor exchange needs every rank on one host");
    return vcclInvalidUsage;
  }
  const uint64_t seq = fdSeq_++;
  int lfd = -1;
  VTRY(unixListen(fdSocketName(rank_, seq), &lfd));
  vcclResult_t res = barrier();  // every listener exists before anyone connects
  // Connect-and-send never blocks: the backlog and socket buffer absorb the
  // small messages, so all ranks may send before anyone accepts.
  for (int s = 1; res == vcclSuccess && s < nranks_; s++) {
    int peer = (rank_ + s) % nranks_;
    int c = -1;
    res = unixConnect(fdSocketName(peer, seq), connectWindowMs(), &c);
    if (res != vcclSuccess) break;
    int32_t hdr[2] = {rank_, static_cast<int32_t>(mine.size())};
    res = sendWithFds(c, hdr, sizeof(hdr), mine);
    closeFd(c);
  }
  for (int s = 1; res == vcclSuccess && s < nranks_; s++) {
    int c = -1;
    res = tcpAccept(lfd, &aborted_, &c);  // accept() works on any stream socket
    if (res != vcclSuccess) break;
    int32_t hdr[2] = {-1, 0};
    std::vector<int> got;
    res = recvWithFds(c, hdr, sizeof(hdr), mine.size() + 1, &got);
    closeFd(c);
    if (res == vcclSuccess &&
        (hdr[0] < 0 || hdr[0] >= nranks_ || hdr[0] == rank_ ||
         got.size() != mine.size() || !(*out)[hdr[0]].empty())) {
      VERR("descriptor exchange: malformed message from rank %d", hdr[0]);
      for (int fd : got) closeFd(fd);
      res = vcclInternalError;
    }
    if (res == vcclSuccess) (*out)[hdr[0]] = got;
  }
  closeFd(lfd);
  if (res == vcclSuccess) res = barrier();
  if (res != vcclSuccess) {
    for (auto& v : *out)
      for (int fd : v) closeFd(fd);
    out->clear();
  }
  return res;
}

vcclResult_t Bootstrap::broadcastFds(int root, std::vector<int>* fds, size_t count) {
  std::vector<int> mine = (rank_ == root) ? *fds : std::vector<int>();
  if (rank_ != root) {
    // Every rank must contribute the same count; non-roots send placeholders.
    for (size_t i = 0; i < count; i++) mine.push_back(dup(STDERR_FILENO));
  }
  std::vector<std::vector<int>> all;
  vcclResult_t res = exchangeFds(mine, &all);
  if (rank_ != root)
    for (int fd : mine) closeFd(fd);
  if (res != vcclSuccess) return res;
  for (int p = 0; p < nranks_; p++) {
    if (p == root) continue;
    for (int fd : all[p]) closeFd(fd);
  }
  if (rank_ == root) {
    for (int fd : all[root]) closeFd(fd);  // dups of our own
  } else {
    *fds = all[root];
  }
  return vcclSuccess;
}

}  // namespace vccl
