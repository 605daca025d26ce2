// SPDX-License-Identifier: Apache-2.0
// Control-plane concurrency test, built without CUDA so it can run under
// ThreadSanitizer / AddressSanitizer on a CPU machine (make sanitize).
//
// Several communicators' bootstraps run as threads of one process: ids made
// concurrently, rendezvous, repeated allGather / broadcast / barrier rounds,
// descriptor exchange over the Unix sockets, and an abort racing a waiting
// rank.  The reference has no sanitizer builds (its concurrency rests on
// documented contracts); this is the race check for the host side that
// replaces its transports.
#include <fcntl.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "control/bootstrap.h"

using vccl::Bootstrap;

namespace {
std::atomic<int> gFail{0};

void check(bool ok, const char* what, int rank) {
  if (!ok) {
    std::fprintf(stderr, "FAIL rank %d: %s\n", rank, what);
    gFail++;
  }
}

void runGroup(int nranks, int rounds) {
  vcclUniqueId id;
  if (vccl::makeUniqueId(&id, false) != vcclSuccess) {
    check(false, "makeUniqueId", -1);
    return;
  }
  std::vector<std::thread> ts;
  for (int r = 0; r < nranks; r++) {
    ts.emplace_back([&, r] {
      std::unique_ptr<Bootstrap> bs;
      check(Bootstrap::create(id, r, nranks, &bs) == vcclSuccess, "create", r);
      if (!bs) return;
      for (int it = 0; it < rounds; it++) {
        std::vector<uint64_t> v(nranks, 0);
        v[r] = 1000u * it + r;
        check(bs->allGather(v.data(), sizeof(uint64_t)) == vcclSuccess, "allGather", r);
        for (int p = 0; p < nranks; p++) check(v[p] == 1000u * it + p, "allGather value", r);
        uint64_t b = r == it % nranks ? 77u + it : 0u;
        check(bs->broadcast(&b, sizeof(b), it % nranks) == vcclSuccess, "broadcast", r);
        check(b == 77u + it, "broadcast value", r);
        check(bs->barrier() == vcclSuccess, "barrier", r);
      }
      // descriptor exchange: every rank sends one pipe end
      int fds[2];
      check(pipe(fds) == 0, "pipe", r);
      std::vector<std::vector<int>> got;
      check(bs->exchangeFds({fds[0]}, &got) == vcclSuccess, "exchangeFds", r);
      check(static_cast<int>(got.size()) == nranks, "exchangeFds count", r);
      for (auto& v : got)
        for (int fd : v) close(fd);
      close(fds[0]);
      close(fds[1]);
    });
  }
  for (auto& t : ts) t.join();
}

// A rank waits in a barrier that can never complete; another thread aborts
// the bootstrap, which must unblock it with an error.
void abortRace() {
  vcclUniqueId id;
  if (vccl::makeUniqueId(&id, false) != vcclSuccess) {
    check(false, "makeUniqueId", -1);
    return;
  }
  std::unique_ptr<Bootstrap> b0, b1;
  std::thread t1([&] { check(Bootstrap::create(id, 1, 2, &b1) == vcclSuccess, "create 1", 1); });
  check(Bootstrap::create(id, 0, 2, &b0) == vcclSuccess, "create 0", 0);
  t1.join();
  if (!b0 || !b1) return;
  std::atomic<bool> returned{false};
  std::thread waiter([&] {
    const vcclResult_t r = b0->barrier();  // rank 1 never joins this barrier
    check(r != vcclSuccess, "barrier after abort must fail", 0);
    returned = true;
  });
  std::this_thread::sleep_for(std::chrono::milliseconds(100));
  b0->abort();
  waiter.join();
  check(returned.load(), "abort unblocks", 0);
}
}  // namespace

int main() {
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 1);
  setenv("VCCL_TIMEOUT", "20", 1);
  // two communicators at once, like a job creating its TP and DP groups
  std::thread g1([] { runGroup(4, 20); });
  std::thread g2([] { runGroup(3, 20); });
  g1.join();
  g2.join();
  abortRace();
  std::printf("bootstrap-threads: %s\n", gFail == 0 ? "OK" : "FAIL");
  return gFail == 0 ? 0 : 1;
}
