// SPDX-License-Identifier: Apache-2.0
// Host data plane concurrency test, built without the CUDA runtime so it can
// run under ThreadSanitizer / AddressSanitizer on a CPU machine (make
// sanitize).
//
// The ranks of one communicator run as threads of one process, each with its
// own bootstrap and TCP mesh.  Large batches hand their sends to the sender
// thread (VCCL_HOST_SEND_THREAD_MIN is set low), so its hand-off and the
// progress loop run under the sanitizers: all-reduce of several sizes and
// types (direct, pipelined in pieces, in place), reduce-scatter, all-gather,
// broadcast (direct and in pieces), reduce, all-to-all(v); then an abort from
// another thread while one rank's large all-reduce waits for a peer that
// never joins.  Results are checked exactly against a rank-order oracle.
#include <cuda_bf16.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "control/bootstrap.h"
#include "runtime/hostplane.h"

using vccl::Bootstrap;
using vccl::HostPlane;
using vccl::HostRed;

namespace {
std::atomic<int> gFail{0};

void check(bool ok, const char* what, int rank) {
  if (!ok) {
    std::fprintf(stderr, "FAIL rank %d: %s\n", rank, what);
    gFail++;
  }
}

// Small integers: every partial sum is exact in f32 and bf16.
float val(int rank, size_t i) { return static_cast<float>((rank * 7 + static_cast<int>(i % 13)) % 9) - 4.0f; }

HostRed sumOf(vcclDataType_t dt) { return HostRed{dt, 0, false, false, 1.0}; }

void rankBody(const vcclUniqueId& id, int rank, int n) {
  std::unique_ptr<Bootstrap> bs;
  if (Bootstrap::create(id, rank, n, &bs) != vcclSuccess) {
    check(false, "bootstrap", rank);
    return;
  }
  std::unique_ptr<HostPlane> hp;
  if (HostPlane::create(bs.get(), &hp) != vcclSuccess) {
    check(false, "host plane", rank);
    return;
  }
  // all-reduce f32: direct (small), pipelined in pieces (large), in place
  for (size_t count : {size_t{5}, size_t{3000}, size_t{1} << 20}) {
    std::vector<float> in(count), out(count, -99.0f);
    for (size_t i = 0; i < count; i++) in[i] = val(rank, i);
    check(hp->allReduce(reinterpret_cast<const char*>(in.data()), reinterpret_cast<char*>(out.data()), count,
                        sumOf(vcclFloat32)) == vcclSuccess,
          "allReduce f32", rank);
    bool ok = true;
    for (size_t i = 0; i < count; i++) {
      float want = 0;
      for (int r = 0; r < n; r++) want += val(r, i);
      ok &= out[i] == want;
    }
    check(ok, "allReduce f32 values", rank);
    check(hp->allReduce(reinterpret_cast<const char*>(in.data()), reinterpret_cast<char*>(in.data()), count,
                        sumOf(vcclFloat32)) == vcclSuccess &&
              std::memcmp(in.data(), out.data(), count * 4) == 0,
          "allReduce f32 in place", rank);
  }
  // all-reduce bf16 (fp32 accumulation, one rounding)
  {
    const size_t count = size_t{1} << 19;
    std::vector<__nv_bfloat16> in(count), out(count);
    for (size_t i = 0; i < count; i++) in[i] = __float2bfloat16_rn(val(rank, i));
    check(hp->allReduce(reinterpret_cast<const char*>(in.data()), reinterpret_cast<char*>(out.data()), count,
                        sumOf(vcclBfloat16)) == vcclSuccess,
          "allReduce bf16", rank);
    bool ok = true;
    for (size_t i = 0; i < count; i++) {
      float want = 0;
      for (int r = 0; r < n; r++) want += val(r, i);
      ok &= __bfloat162float(out[i]) == want;
    }
    check(ok, "allReduce bf16 values", rank);
  }
  // reduce-scatter and all-gather
  {
    const size_t per = (size_t{1} << 18) + 3;
    std::vector<float> in(per * n), out(per);
    for (size_t i = 0; i < in.size(); i++) in[i] = val(rank, i);
    check(hp->reduceScatter(reinterpret_cast<const char*>(in.data()), reinterpret_cast<char*>(out.data()), per,
                            sumOf(vcclFloat32)) == vcclSuccess,
          "reduceScatter", rank);
    bool ok = true;
    for (size_t i = 0; i < per; i++) {
      float want = 0;
      for (int r = 0; r < n; r++) want += val(r, rank * per + i);
      ok &= out[i] == want;
    }
    check(ok, "reduceScatter values", rank);
    std::vector<float> all(per * n, -1.0f);
    check(hp->allGather(reinterpret_cast<const char*>(out.data()), reinterpret_cast<char*>(all.data()),
                        per * 4) == vcclSuccess,
          "allGather", rank);
    ok = true;
    for (size_t i = 0; i < all.size(); i++) {
      float want = 0;
      for (int r = 0; r < n; r++) want += val(r, i);
      ok &= all[i] == want;
    }
    check(ok, "allGather values", rank);
  }
  // broadcast (direct and in pieces) and reduce, every root
  for (int root = 0; root < n; root++) {
    for (size_t bytes : {size_t{1000}, size_t{3} << 20}) {
      std::vector<char> b(bytes);
      for (size_t i = 0; i < bytes; i++) b[i] = rank == root ? static_cast<char>(i * 31 + root) : 0;
      check(hp->broadcast(b.data(), b.data(), bytes, root) == vcclSuccess, "broadcast", rank);
      bool ok = true;
      for (size_t i = 0; i < bytes; i++) ok &= b[i] == static_cast<char>(i * 31 + root);
      check(ok, "broadcast values", rank);
    }
    const size_t count = size_t{1} << 18;
    std::vector<float> in(count), out(count, 0.0f);
    for (size_t i = 0; i < count; i++) in[i] = val(rank, i);
    check(hp->reduce(reinterpret_cast<const char*>(in.data()), reinterpret_cast<char*>(out.data()), count,
                     sumOf(vcclFloat32), root) == vcclSuccess,
          "reduce", rank);
    if (rank == root) {
      bool ok = true;
      for (size_t i = 0; i < count; i++) {
        float want = 0;
        for (int r = 0; r < n; r++) want += val(r, i);
        ok &= out[i] == want;
      }
      check(ok, "reduce values", rank);
    }
  }
  // all-to-all(v): rank r sends (r + p + 1) * 4096 bytes to rank p
  {
    std::vector<size_t> sc(n), sd(n), rc(n), rd(n);
    size_t st = 0, rt = 0;
    for (int p = 0; p < n; p++) {
      sc[p] = static_cast<size_t>(rank + p + 1) * 4096;
      sd[p] = st;
      st += sc[p];
      rc[p] = static_cast<size_t>(p + rank + 1) * 4096;
      rd[p] = rt;
      rt += rc[p];
    }
    std::vector<unsigned char> s(st), r(rt, 0);
    for (int p = 0; p < n; p++)
      for (size_t i = 0; i < sc[p]; i++) s[sd[p] + i] = static_cast<unsigned char>(rank * 16 + p + i);
    check(hp->allToAllv(reinterpret_cast<const char*>(s.data()), sc.data(), sd.data(),
                        reinterpret_cast<char*>(r.data()), rc.data(), rd.data()) == vcclSuccess,
          "allToAllv", rank);
    bool ok = true;
    for (int p = 0; p < n; p++)
      for (size_t i = 0; i < rc[p]; i++) ok &= r[rd[p] + i] == static_cast<unsigned char>(p * 16 + rank + i);
    check(ok, "allToAllv values", rank);
  }
  check(bs->barrier() == vcclSuccess, "final barrier", rank);
}

void runGroup(int n) {
  vcclUniqueId id;
  if (vccl::makeUniqueId(&id, false) != vcclSuccess) {
    check(false, "makeUniqueId", -1);
    return;
  }
  std::vector<std::thread> ts;
  for (int r = 0; r < n; r++) ts.emplace_back([&id, r, n] { rankBody(id, r, n); });
  for (auto& t : ts) t.join();
}

// Rank 0 starts a 16 MiB all-reduce that rank 1 never joins; an abort from a
// third thread must end it (both the receive loop and the sender thread).
void abortRace() {
  vcclUniqueId id;
  if (vccl::makeUniqueId(&id, false) != vcclSuccess) {
    check(false, "makeUniqueId", -1);
    return;
  }
  std::unique_ptr<HostPlane> planes[2];
  std::unique_ptr<Bootstrap> boots[2];
  std::thread mk[2];
  for (int r = 0; r < 2; r++)
    mk[r] = std::thread([&, r] {
      check(Bootstrap::create(id, r, 2, &boots[r]) == vcclSuccess, "bootstrap", r);
      if (boots[r]) check(HostPlane::create(boots[r].get(), &planes[r]) == vcclSuccess, "host plane", r);
    });
  for (auto& t : mk) t.join();
  if (!planes[0] || !planes[1]) return;
  const size_t count = size_t{1} << 22;
  std::vector<float> in(count, 1.0f), out(count);
  std::atomic<bool> returned{false};
  vcclResult_t res = vcclSuccess;
  std::thread waiter([&] {
    res = planes[0]->allReduce(reinterpret_cast<const char*>(in.data()), reinterpret_cast<char*>(out.data()), count,
                               sumOf(vcclFloat32));
    returned = true;
  });
  std::this_thread::sleep_for(std::chrono::milliseconds(300));
  check(!returned.load(), "all-reduce waits for the missing peer", 0);
  planes[0]->abort();
  waiter.join();
  check(returned.load() && res != vcclSuccess, "abort ends the all-reduce with an error", 0);
}
}  // namespace

int main() {
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 1);
  setenv("VCCL_TIMEOUT", "30", 1);
  setenv("VCCL_HOST_SEND_THREAD_MIN", "4096", 1);  // most batches use the sender thread
  setenv("VCCL_HOST_CHUNK", "65536", 1);           // many pipelined pieces
  setenv("VCCL_HOST_BCAST_PIECE", "65536", 1);
  // two communicators at once
  std::thread g1([] { runGroup(3); });
  std::thread g2([] { runGroup(2); });
  g1.join();
  g2.join();
  abortRace();
  std::printf("hostplane-threads: %s\n", gFail == 0 ? "OK" : "FAIL");
  return gFail == 0 ? 0 : 1;
}
