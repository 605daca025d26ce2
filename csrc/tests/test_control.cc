// SPDX-License-Identifier: Apache-2.0
// Control-plane suite (CPU only; VCCL_NO_DEVICE=1 forces control-plane
// communicators even on GPU machines).  Mirrors the parts of the reference's
// suite that need no data plane (reference: tests/test_collectives.cc:
// 355-466 PreMulSum / split / misc, :542-612 kill-a-rank, :618-647 InitAll).
//
// Covers what needs no data plane: error strings and type sizes, version,
// group nesting rules, init / split (even-odd and NOCOLOR) / InitAll
// membership, VCCL_COMM_ID-derived ids, PreMulSum op table (slot reuse,
// float-only, rejection after destroy), abort latch and async error,
// MemAlloc host fallback with double-free rejection, single-rank host
// collectives, and failure detection without a GPU: a rank that never
// joins makes the others' init fail within VCCL_TIMEOUT, and a rank that
// dies makes the survivors' next collective control step (split) fail.
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "vccl.h"

namespace {

int gFail = 0;
#define EXPECT(c, ...)                                                 \
  do {                                                                 \
    if (!(c)) {                                                        \
      std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__);        \
      std::fprintf(stderr, __VA_ARGS__);                               \
      std::fprintf(stderr, "\n");                                      \
      gFail++;                                                         \
    }                                                                  \
  } while (0)

template <typename F>
int forkEach(int n, F&& body) {
  std::vector<pid_t> pids;
  for (int r = 0; r < n; r++) {
    pid_t p = fork();
    if (p == 0) _exit(body(r));
    pids.push_back(p);
  }
  int bad = 0;
  for (pid_t p : pids) {
    int st = 0;
    waitpid(p, &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) bad++;
  }
  return bad;
}

void basics() {
  EXPECT(std::strcmp(vcclGetErrorString(vcclSuccess), "no error") == 0, "error string");
  EXPECT(std::strcmp(vcclGetErrorString(vcclRemoteError), "remote process error") == 0, "error string");
  EXPECT(vcclTypeSize(vcclBfloat16) == 2 && vcclTypeSize(vcclFloat64) == 8 && vcclTypeSize(vcclInt8) == 1 &&
             vcclTypeSize(vcclFloat8e4m3) == 1 && vcclTypeSize(static_cast<vcclDataType_t>(99)) == 0,
         "type sizes");
  int v = 0;
  EXPECT(vcclGetVersion(&v) == vcclSuccess && v == VCCL_VERSION_CODE, "version");
  EXPECT(vcclGetVersion(nullptr) == vcclInvalidArgument, "null version");
  EXPECT(vcclGroupEnd() == vcclInvalidUsage, "unbalanced GroupEnd accepted");
  EXPECT(vcclGroupStart() == vcclSuccess && vcclGroupStart() == vcclSuccess, "nested start");
  EXPECT(vcclGroupEnd() == vcclSuccess && vcclGroupEnd() == vcclSuccess, "nested end");
  vcclConfig_t bad{1, 1, 0};
  vcclComm_t c = nullptr;
  vcclUniqueId id{};
  EXPECT(vcclCommInitRankConfig(&c, 1, id, 0, &bad) == vcclInvalidArgument, "bad config accepted");
  EXPECT(vcclCommInitRank(&c, 1, id, 0) == vcclInvalidArgument, "garbage id accepted");
  EXPECT(vcclCommInitRank(&c, 2, id, 2) == vcclInvalidArgument, "rank out of range accepted");
}

void memory() {
  void* p = nullptr;
  EXPECT(vcclMemAlloc(&p, 5000) == vcclSuccess && p != nullptr, "memalloc");
  std::memset(p, 0xab, 5000);
  EXPECT(vcclMemFree(p) == vcclSuccess, "memfree");
  EXPECT(vcclMemFree(p) == vcclInvalidArgument, "double free accepted");
  EXPECT(vcclMemFree(nullptr) == vcclSuccess, "free(NULL)");
}

void singleRank() {
  vcclUniqueId id;
  vcclComm_t c = nullptr;
  EXPECT(vcclGetUniqueId(&id) == vcclSuccess, "uid");
  EXPECT(vcclCommInitRank(&c, 1, id, 0) == vcclSuccess, "init 1");
  if (!c) return;
  int dev = 0;
  vcclCommDevice(c, &dev);
  EXPECT(dev == -1, "control-plane comm reports device %d", dev);
  std::vector<float> a(17), b(17, -1.0f);
  for (int i = 0; i < 17; i++) a[i] = static_cast<float>(i);
  EXPECT(vcclAllReduce(a.data(), b.data(), 17, vcclFloat32, vcclSum, c) == vcclSuccess && b[16] == 16.0f, "1-rank AR");
  EXPECT(vcclAllGather(a.data(), b.data(), 17, vcclFloat32, c) == vcclSuccess && b[3] == 3.0f, "1-rank AG");
  float k = 3.0f;
  vcclRedOp_t op;
  EXPECT(vcclRedOpCreatePreMulSum(&op, &k, vcclFloat32, vcclScalarHostImmediate, c) == vcclSuccess, "premul");
  EXPECT(op == vcclNumOps, "first custom op value %d", op);
  EXPECT(vcclAllReduce(a.data(), b.data(), 17, vcclFloat32, op, c) == vcclSuccess && b[2] == 6.0f, "premul AR");
  EXPECT(vcclAllReduce(a.data(), b.data(), 17, vcclInt32, op, c) == vcclInvalidArgument, "premul on int accepted");
  EXPECT(vcclAllReduce(a.data(), b.data(), 17, vcclInt32, vcclAvg, c) == vcclInvalidArgument, "avg on int accepted");
  vcclRedOp_t op2;
  EXPECT(vcclRedOpCreatePreMulSum(&op2, &k, vcclInt32, vcclScalarHostImmediate, c) == vcclInvalidArgument,
         "int scalar accepted");
  EXPECT(vcclRedOpCreatePreMulSum(&op2, &k, vcclFloat32, vcclScalarDevice, c) == vcclInvalidArgument,
         "device scalar accepted");
  EXPECT(vcclRedOpDestroy(op, c) == vcclSuccess, "destroy op");
  EXPECT(vcclRedOpDestroy(op, c) == vcclInvalidArgument, "double destroy accepted");
  EXPECT(vcclAllReduce(a.data(), b.data(), 17, vcclFloat32, op, c) == vcclInvalidArgument, "destroyed op accepted");
  EXPECT(vcclRedOpCreatePreMulSum(&op2, &k, vcclFloat32, vcclScalarHostImmediate, c) == vcclSuccess && op2 == op,
         "freed slot not reused");
  EXPECT(vcclSend(a.data(), 1, vcclFloat32, 0, c) == vcclInvalidArgument, "send to self accepted");
  EXPECT(vcclBroadcast(a.data(), b.data(), 4, vcclFloat32, 3, c) == vcclInvalidArgument, "bad root accepted");
  EXPECT(vcclCommAbort(c) == vcclSuccess, "abort");
  EXPECT(vcclAllReduce(a.data(), b.data(), 17, vcclFloat32, vcclSum, c) == vcclInvalidUsage, "aborted comm usable");
  vcclResult_t ae = vcclSuccess;
  EXPECT(vcclCommGetAsyncError(c, &ae) == vcclSuccess && ae != vcclSuccess, "async error after abort");
  EXPECT(vcclCommDestroy(c) == vcclSuccess, "destroy");
}

int splitRank(int r, int n, const vcclUniqueId& id) {
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, n, id, r) != vcclSuccess) return 1;
  vcclComm_t s = nullptr;
  // Reverse key order inside each color: new rank = reversed position.
  if (vcclCommSplit(c, r % 2, -r, &s, nullptr) != vcclSuccess || s == nullptr) return 2;
  int sr = -1, sn = -1;
  vcclCommUserRank(s, &sr);
  vcclCommCount(s, &sn);
  const int members = (n + (r % 2 == 0 ? 1 : 0)) / 2;
  const int want = members - 1 - r / 2;
  if (sn != members || sr != want) {
    std::fprintf(stderr, "rank %d: split got %d/%d want %d/%d\n", r, sr, sn, want, members);
    return 3;
  }
  vcclCommDestroy(s);
  vcclComm_t s2 = nullptr;
  if (vcclCommSplit(c, r == 0 ? VCCL_SPLIT_NOCOLOR : 3, 0, &s2, nullptr) != vcclSuccess) return 4;
  if ((r == 0) != (s2 == nullptr)) return 5;
  if (s2) {
    int cnt = 0;
    vcclCommCount(s2, &cnt);
    if (cnt != n - 1) return 6;
    vcclCommDestroy(s2);
  }
  // Without a device, host buffers move over the host data plane (TCP mesh).
  std::vector<float> x(4, 1.0f + r);
  if (vcclAllReduce(x.data(), x.data(), 4, vcclFloat32, vcclSum, c) != vcclSuccess) return 7;
  const float sum = n + n * (n - 1) / 2.0f;
  for (float v : x)
    if (v != sum) return 8;
  vcclCommDestroy(c);
  return 0;
}

void commIdEnv() {
  // Every rank derives the id locally; rank 0 binds the port at init.
  setenv("VCCL_COMM_ID", "127.0.0.1:41917", 1);
  int bad = forkEach(3, [](int r) {
    vcclUniqueId id;
    if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
    vcclComm_t c = nullptr;
    if (vcclCommInitRank(&c, 3, id, r) != vcclSuccess) return 2;
    int n = 0;
    vcclCommCount(c, &n);
    vcclCommDestroy(c);
    return n == 3 ? 0 : 3;
  });
  unsetenv("VCCL_COMM_ID");
  EXPECT(bad == 0, "VCCL_COMM_ID rendezvous failed on %d ranks", bad);
}

void initAll() {
  std::vector<vcclComm_t> c(3, nullptr);
  EXPECT(vcclCommInitAll(c.data(), 3, nullptr) == vcclSuccess, "InitAll");
  for (int i = 0; i < 3; i++) {
    int r = -1, n = -1;
    if (!c[i]) continue;
    vcclCommUserRank(c[i], &r);
    vcclCommCount(c[i], &n);
    EXPECT(r == i && n == 3, "InitAll comm %d: %d/%d", i, r, n);
  }
  // One thread drives all three ranks inside a group: the host data plane
  // runs each communicator's calls on its own thread so the ranks meet.
  if (c[0] && c[1] && c[2]) {
    std::vector<std::vector<double>> x(3, std::vector<double>(5000));
    std::vector<std::vector<int32_t>> g(3, std::vector<int32_t>(3 * 7));
    std::vector<int32_t> mine[3];
    for (int i = 0; i < 3; i++) {
      for (size_t k = 0; k < x[i].size(); k++) x[i][k] = i + 0.5 * k;
      mine[i].assign(7, 100 * i);
    }
    vcclGroupStart();
    for (int i = 0; i < 3; i++) {
      vcclAllReduce(x[i].data(), x[i].data(), x[i].size(), vcclFloat64, vcclSum, c[i]);
      vcclAllGather(mine[i].data(), g[i].data(), 7, vcclInt32, c[i]);
    }
    EXPECT(vcclGroupEnd() == vcclSuccess, "InitAll group of host collectives");
    for (int i = 0; i < 3; i++) {
      for (size_t k = 0; k < x[i].size(); k++)
        if (x[i][k] != 3 + 1.5 * k) {
          EXPECT(false, "InitAll all-reduce rank %d [%zu] = %g", i, k, x[i][k]);
          break;
        }
      for (int p = 0; p < 3; p++)
        EXPECT(g[i][p * 7] == 100 * p && g[i][p * 7 + 6] == 100 * p, "InitAll all-gather rank %d block %d", i, p);
    }
  }
  for (int i = 0; i < 3; i++)
    if (c[i]) vcclCommDestroy(c[i]);
}

// Failure detection on the host: a missing rank must not hang the others.
void missingRank() {
  setenv("VCCL_TIMEOUT", "2", 1);
  vcclUniqueId id;
  vcclGetUniqueId(&id);
  auto t0 = std::chrono::steady_clock::now();
  int bad = forkEach(2, [&](int r) {
    vcclComm_t c = nullptr;
    vcclResult_t res = vcclCommInitRank(&c, 3, id, r);  // rank 2 never joins
    return res == vcclSystemError ? 0 : 1;
  });
  const long secs = std::chrono::duration_cast<std::chrono::seconds>(std::chrono::steady_clock::now() - t0).count();
  EXPECT(bad == 0, "missing rank: %d ranks did not report vcclSystemError", bad);
  EXPECT(secs < 20, "missing rank took %lds (hang?)", secs);
  unsetenv("VCCL_TIMEOUT");
}

void deadPeer() {
  setenv("VCCL_TIMEOUT", "2", 1);
  vcclUniqueId id;
  vcclGetUniqueId(&id);
  int bad = forkEach(3, [&](int r) {
    vcclComm_t c = nullptr;
    if (vcclCommInitRank(&c, 3, id, r) != vcclSuccess) return 1;
    if (r == 1) _exit(0);  // leaves between steps
    usleep(200 * 1000);
    vcclComm_t s = nullptr;
    vcclResult_t res = vcclCommSplit(c, 0, r, &s, nullptr);
    return res != vcclSuccess ? 0 : 2;
  });
  EXPECT(bad == 0, "dead peer: survivors' split did not fail (%d)", bad);
  unsetenv("VCCL_TIMEOUT");
}

}  // namespace

int main() {
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
  setenv("VCCL_NO_DEVICE", "1", 1);
  basics();
  memory();
  singleRank();
  for (int n : {2, 3, 5}) {
    vcclUniqueId id;
    vcclGetUniqueId(&id);
    int bad = forkEach(n, [&](int r) { return splitRank(r, n, id); });
    EXPECT(bad == 0, "split with %d ranks: %d failures", n, bad);
  }
  commIdEnv();
  initAll();
  missingRank();
  deadPeer();
  std::printf("control-plane: %s\n", gFail ? "FAIL" : "OK");
  return gFail ? 1 : 0;
}
