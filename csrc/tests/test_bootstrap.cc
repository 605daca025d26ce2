// SPDX-License-Identifier: Apache-2.0
// Rendezvous hardening: a stray client with a wrong rank count connects to
// the root first and must be rejected with an explicit reply, after which
// the root keeps listening and the real two-rank job still forms.  Same
// scenario as the reference's test (reference: tests/test_bootstrap.cc:
// 41-105); runs on the CPU (no device needed).
#include <sys/wait.h>
#include <unistd.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common/net.h"
#include "control/bootstrap.h"
#include "vccl.h"

namespace {

// Wire copy of the 48-byte join record sent by every non-root rank.
struct Join {
  uint32_t magic;
  uint32_t version;
  uint64_t nonce;
  int32_t nranks;
  int32_t rank;
  uint32_t orderTag;
  int32_t reserved;
  uint64_t hostHash;
  int32_t pid;
  int32_t device;
};
static_assert(sizeof(Join) == 48, "join layout");

int strayClient(const vcclUniqueId& uid) {
  vccl::IdLayout id;
  std::memcpy(&id, uid.internal, sizeof(id));
  int fd = -1;
  if (vccl::tcpConnect(id.root, 3000, &fd) != vcclSuccess) return 2;
  Join j{};
  j.magic = id.magic;
  j.version = VCCL_VERSION_CODE;
  j.nonce = id.nonce;
  j.nranks = 99;  // wrong: the job has two ranks
  j.rank = 1;
  j.orderTag = 0x01020304u;
  if (vccl::sendFull(fd, &j, sizeof(j)) != vcclSuccess) return 3;
  uint8_t verdict = 0xff;
  vcclResult_t r = vccl::recvFull(fd, &verdict, 1);
  vccl::closeFd(fd);
  return (r == vcclSuccess && verdict == 0) ? 0 : 1;
}

int realRank(int rank, const vcclUniqueId& id) {
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, 2, id, rank) != vcclSuccess || c == nullptr) return 1;
  int r = -1, n = -1;
  vcclCommUserRank(c, &r);
  vcclCommCount(c, &n);
  vcclCommDestroy(c);
  return (r == rank && n == 2) ? 0 : 1;
}

}  // namespace

int main() {
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
  setenv("VCCL_TIMEOUT", "10", 1);
  setenv("VCCL_NO_DEVICE", "1", 1);
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) {
    std::printf("bootstrap-reject: FAIL (unique id)\n");
    return 1;
  }
  pid_t root = fork();
  if (root == 0) _exit(realRank(0, id));
  const int stray = strayClient(id);
  pid_t peer = fork();
  if (peer == 0) _exit(realRank(1, id));
  int s0 = 0, s1 = 0;
  waitpid(root, &s0, 0);
  waitpid(peer, &s1, 0);
  const bool ok = stray == 0 && WIFEXITED(s0) && WEXITSTATUS(s0) == 0 && WIFEXITED(s1) && WEXITSTATUS(s1) == 0;
  if (!ok) std::fprintf(stderr, "stray=%d root=%d peer=%d\n", stray, WEXITSTATUS(s0), WEXITSTATUS(s1));
  std::printf("bootstrap-reject: %s\n", ok ? "OK" : "FAIL");
  return ok ? 0 : 1;
}
