// SPDX-License-Identifier: Apache-2.0
// Multi-process correctness suite on GPUs.
//
// Same coverage as the reference's fork-based suite (reference:
// tests/test_collectives.cc:468-612): all-gather, reduce-scatter and
// all-reduce (sum/max/min over f32/f16/bf16/i32/f64, in place and out of
// place) at counts {1, 7, 1024, 65539}; avg; reduce and broadcast from every
// root; send/recv pairs; grouped send/recv with both neighbours; gather and
// scatter; all-to-all and uneven all-to-allv; PreMulSum and its rejection
// after destroy; split with NOCOLOR; misc (version, device, async error,
// finalize, MemAlloc + Register + all-reduce, double free, Bcast); forced
// algorithm A/B; kill-a-rank; InitAll.  Ranks are forked processes, one GPU
// each.  Buffers are host std::vectors (the staged path) and, for the
// additions, device buffers at sizes that reach every algorithm.
//
// Usage: test_collectives [maxRanks]   (default: number of visible GPUs)
#include <cuda_runtime.h>
#include <sys/wait.h>
#include <unistd.h>

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "vccl.h"
#include "vccl_x.h"

namespace {

int gFail = 0;

#define EXPECT(cond, ...)                                   \
  do {                                                      \
    if (!(cond)) {                                          \
      std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      std::fprintf(stderr, __VA_ARGS__);                    \
      std::fprintf(stderr, "\n");                           \
      gFail++;                                              \
    }                                                       \
  } while (0)
#define EXPECT_OK(call) EXPECT((call) == vcclSuccess, "%s -> %s", #call, vcclGetLastError(nullptr))

// Small integers keep f16/bf16 sums exact.
float val(int rank, size_t i) { return static_cast<float>((rank * 13 + i * 5) % 16); }

uint16_t toHalf(float f) {  // exact for the small integers used here
  if (f == 0.0f) return 0;
  int e;
  float m = std::frexp(f, &e);  // f = m * 2^e, m in [0.5,1)
  uint32_t mant = static_cast<uint32_t>((m * 2.0f - 1.0f) * 1024.0f + 0.5f);
  return static_cast<uint16_t>(((e - 1 + 15) << 10) | mant);
}
float fromHalf(uint16_t h) {
  if ((h & 0x7fff) == 0) return 0.0f;
  int e = (h >> 10) & 0x1f;
  float m = 1.0f + (h & 0x3ff) / 1024.0f;
  float v = std::ldexp(m, e - 15);
  return (h & 0x8000) ? -v : v;
}
uint16_t toBf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return static_cast<uint16_t>(u >> 16);
}
float fromBf16(uint16_t b) {
  uint32_t u = static_cast<uint32_t>(b) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

void put(void* buf, vcclDataType_t dt, size_t i, float v) {
  switch (dt) {
    case vcclFloat32: static_cast<float*>(buf)[i] = v; break;
    case vcclFloat64: static_cast<double*>(buf)[i] = v; break;
    case vcclInt32: static_cast<int32_t*>(buf)[i] = static_cast<int32_t>(v); break;
    case vcclFloat16: static_cast<uint16_t*>(buf)[i] = toHalf(v); break;
    case vcclBfloat16: static_cast<uint16_t*>(buf)[i] = toBf16(v); break;
    default: std::abort();
  }
}
float get(const void* buf, vcclDataType_t dt, size_t i) {
  switch (dt) {
    case vcclFloat32: return static_cast<const float*>(buf)[i];
    case vcclFloat64: return static_cast<float>(static_cast<const double*>(buf)[i]);
    case vcclInt32: return static_cast<float>(static_cast<const int32_t*>(buf)[i]);
    case vcclFloat16: return fromHalf(static_cast<const uint16_t*>(buf)[i]);
    case vcclBfloat16: return fromBf16(static_cast<const uint16_t*>(buf)[i]);
    default: std::abort();
  }
}
void fill(void* buf, vcclDataType_t dt, int rank, size_t n, size_t off = 0) {
  for (size_t i = 0; i < n; i++) put(buf, dt, i, val(rank, off + i));
}

float expect(vcclRedOp_t op, int n, size_t i) {
  float a = val(0, i);
  for (int r = 1; r < n; r++) {
    float b = val(r, i);
    if (op == vcclSum || op == vcclAvg) a += b;
    else if (op == vcclProd) a *= b;
    else if (op == vcclMax) a = a > b ? a : b;
    else if (op == vcclMin) a = a < b ? a : b;
  }
  return op == vcclAvg ? a / n : a;
}

bool near(float got, float want, vcclDataType_t dt) {
  float tol = std::fabs(want) * 1e-6f + 1e-6f;
  if (dt == vcclFloat16) tol = std::fabs(want) * 1e-2f + 1e-3f;
  if (dt == vcclBfloat16) tol = std::fabs(want) * 4e-2f + 1e-2f;
  return std::fabs(got - want) <= tol;
}

#define EXPECT_NEAR(got, want, dt, what, idx)                                              \
  do {                                                                                     \
    float g_ = (got), w_ = (want);                                                          \
    if (!near(g_, w_, dt)) {                                                               \
      std::fprintf(stderr, "FAIL %s:%d: %s[%zu]: got %g want %g\n", __FILE__, __LINE__, what, \
                   static_cast<size_t>(idx), g_, w_);                                       \
      gFail++;                                                                              \
      return;                                                                               \
    }                                                                                      \
  } while (0)

void allGather(vcclComm_t c, int me, int n, vcclDataType_t dt, size_t cnt) {
  const size_t es = vcclTypeSize(dt);
  std::vector<char> s(cnt * es), r(n * cnt * es), r2(n * cnt * es);
  fill(s.data(), dt, me, cnt);
  EXPECT_OK(vcclAllGather(s.data(), r.data(), cnt, dt, c));
  for (int p = 0; p < n; p++)
    for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(get(r.data(), dt, p * cnt + i), val(p, i), dt, "allgather", i);
  fill(r2.data() + me * cnt * es, dt, me, cnt);
  EXPECT_OK(vcclAllGather(r2.data() + me * cnt * es, r2.data(), cnt, dt, c));
  EXPECT(std::memcmp(r.data(), r2.data(), r.size()) == 0, "allgather in-place mismatch");
}

void reduceScatter(vcclComm_t c, int me, int n, vcclDataType_t dt, vcclRedOp_t op, size_t rc) {
  const size_t es = vcclTypeSize(dt);
  std::vector<char> s(n * rc * es), r(rc * es);
  fill(s.data(), dt, me, n * rc);
  EXPECT_OK(vcclReduceScatter(s.data(), r.data(), rc, dt, op, c));
  for (size_t i = 0; i < rc; i++) EXPECT_NEAR(get(r.data(), dt, i), expect(op, n, me * rc + i), dt, "reducescatter", i);
  // in place
  EXPECT_OK(vcclReduceScatter(s.data(), s.data() + me * rc * es, rc, dt, op, c));
  EXPECT(std::memcmp(s.data() + me * rc * es, r.data(), r.size()) == 0, "reducescatter in-place mismatch");
}

void allReduce(vcclComm_t c, int me, int n, vcclDataType_t dt, vcclRedOp_t op, size_t cnt) {
  const size_t es = vcclTypeSize(dt);
  std::vector<char> s(cnt * es), r(cnt * es);
  fill(s.data(), dt, me, cnt);
  EXPECT_OK(vcclAllReduce(s.data(), r.data(), cnt, dt, op, c));
  for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(get(r.data(), dt, i), expect(op, n, i), dt, "allreduce", i);
  EXPECT_OK(vcclAllReduce(s.data(), s.data(), cnt, dt, op, c));
  EXPECT(std::memcmp(s.data(), r.data(), r.size()) == 0, "allreduce in-place mismatch");
}

void reduceAll(vcclComm_t c, int me, int n, vcclDataType_t dt, vcclRedOp_t op, size_t cnt) {
  const size_t es = vcclTypeSize(dt);
  for (int root = 0; root < n; root++) {
    std::vector<char> s(cnt * es), r(cnt * es, 0x5a);
    fill(s.data(), dt, me, cnt);
    EXPECT_OK(vcclReduce(s.data(), r.data(), cnt, dt, op, root, c));
    if (me == root)
      for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(get(r.data(), dt, i), expect(op, n, i), dt, "reduce", i);
  }
}

void broadcastAll(vcclComm_t c, int me, int n, size_t cnt) {
  std::vector<float> b(cnt);
  for (int root = 0; root < n; root++) {
    if (me == root) fill(b.data(), vcclFloat32, root, cnt);
    else std::fill(b.begin(), b.end(), -1.0f);
    EXPECT_OK(vcclBroadcast(b.data(), b.data(), cnt, vcclFloat32, root, c));
    for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(b[i], val(root, i), vcclFloat32, "broadcast", i);
  }
}

void sendRecvPairs(vcclComm_t c, int me, int n, size_t cnt) {
  int peer = me ^ 1;
  if (n < 2 || peer >= n) return;
  std::vector<float> mine(cnt), got(cnt, -1.0f);
  fill(mine.data(), vcclFloat32, me, cnt);
  if (me < peer) {
    EXPECT_OK(vcclSend(mine.data(), cnt, vcclFloat32, peer, c));
    EXPECT_OK(vcclRecv(got.data(), cnt, vcclFloat32, peer, c));
  } else {
    EXPECT_OK(vcclRecv(got.data(), cnt, vcclFloat32, peer, c));
    EXPECT_OK(vcclSend(mine.data(), cnt, vcclFloat32, peer, c));
  }
  for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(got[i], val(peer, i), vcclFloat32, "sendrecv", i);
}

void groupNeighbours(vcclComm_t c, int me, int n, size_t cnt) {
  if (n < 2) return;
  const int next = (me + 1) % n, prev = (me + n - 1) % n;
  std::vector<float> toN(cnt), toP(cnt), fromN(cnt, -1), fromP(cnt, -1);
  fill(toN.data(), vcclFloat32, 2 * me, cnt);
  fill(toP.data(), vcclFloat32, 2 * me + 1, cnt);
  EXPECT_OK(vcclGroupStart());
  if (next != prev) {
    EXPECT_OK(vcclSend(toN.data(), cnt, vcclFloat32, next, c));
    EXPECT_OK(vcclSend(toP.data(), cnt, vcclFloat32, prev, c));
    EXPECT_OK(vcclRecv(fromP.data(), cnt, vcclFloat32, prev, c));
    EXPECT_OK(vcclRecv(fromN.data(), cnt, vcclFloat32, next, c));
  } else {
    EXPECT_OK(vcclSend(toN.data(), cnt, vcclFloat32, next, c));
    EXPECT_OK(vcclRecv(fromP.data(), cnt, vcclFloat32, prev, c));
  }
  EXPECT_OK(vcclGroupEnd());
  for (size_t i = 0; i < cnt; i++) {
    EXPECT_NEAR(fromP[i], val(2 * prev, i), vcclFloat32, "group fromPrev", i);
    if (next != prev) EXPECT_NEAR(fromN[i], val(2 * next + 1, i), vcclFloat32, "group fromNext", i);
  }
}

void gatherScatter(vcclComm_t c, int me, int n, size_t cnt) {
  std::vector<float> s(cnt), all(cnt * n, -1.0f), back(cnt, -1.0f);
  fill(s.data(), vcclFloat32, me, cnt);
  const int root = n - 1;
  EXPECT_OK(vcclGather(s.data(), all.data(), cnt, vcclFloat32, root, c));
  if (me == root)
    for (int p = 0; p < n; p++)
      for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(all[p * cnt + i], val(p, i), vcclFloat32, "gather", i);
  EXPECT_OK(vcclScatter(all.data(), back.data(), cnt, vcclFloat32, root, c));
  for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(back[i], val(me, i), vcclFloat32, "scatter", i);
}

void allToAll(vcclComm_t c, int me, int n, size_t cnt) {
  std::vector<float> s(cnt * n), r(cnt * n, -1.0f);
  for (int p = 0; p < n; p++)
    for (size_t i = 0; i < cnt; i++) s[p * cnt + i] = val(me * n + p, i);
  EXPECT_OK(vcclAllToAll(s.data(), r.data(), cnt, vcclFloat32, c));
  for (int p = 0; p < n; p++)
    for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(r[p * cnt + i], val(p * n + me, i), vcclFloat32, "alltoall", i);
  // uneven: rank r sends r+1 elements to every peer
  std::vector<size_t> sc(n, me + 1), sd(n), rc(n), rd(n);
  size_t so = 0, ro = 0;
  for (int p = 0; p < n; p++) {
    sd[p] = so;
    so += sc[p];
    rc[p] = p + 1;
    rd[p] = ro;
    ro += rc[p];
  }
  std::vector<float> vs(so), vr(ro, -1.0f);
  for (int p = 0; p < n; p++)
    for (size_t i = 0; i < sc[p]; i++) vs[sd[p] + i] = static_cast<float>(me * 100 + p);
  EXPECT_OK(vcclAllToAllv(vs.data(), sc.data(), sd.data(), vr.data(), rc.data(), rd.data(), vcclFloat32, c));
  for (int p = 0; p < n; p++)
    for (size_t i = 0; i < rc[p]; i++)
      EXPECT_NEAR(vr[rd[p] + i], static_cast<float>(p * 100 + me), vcclFloat32, "alltoallv", i);
}

void preMulSum(vcclComm_t c, int me, int n, size_t cnt) {
  float k = 0.5f;
  vcclRedOp_t op;
  EXPECT_OK(vcclRedOpCreatePreMulSum(&op, &k, vcclFloat32, vcclScalarHostImmediate, c));
  std::vector<float> s(cnt), r(cnt);
  fill(s.data(), vcclFloat32, me, cnt);
  EXPECT_OK(vcclAllReduce(s.data(), r.data(), cnt, vcclFloat32, op, c));
  for (size_t i = 0; i < cnt; i++) {
    float w = 0;
    for (int p = 0; p < n; p++) w += 0.5f * val(p, i);
    EXPECT_NEAR(r[i], w, vcclFloat32, "premulsum allreduce", i);
  }
  const size_t per = cnt / n;
  if (per > 0) {
    std::vector<float> rs(per);
    EXPECT_OK(vcclReduceScatter(s.data(), rs.data(), per, vcclFloat32, op, c));
    for (size_t i = 0; i < per; i++) {
      float w = 0;
      for (int p = 0; p < n; p++) w += 0.5f * val(p, me * per + i);
      EXPECT_NEAR(rs[i], w, vcclFloat32, "premulsum reducescatter", i);
    }
  }
  EXPECT_OK(vcclRedOpDestroy(op, c));
  EXPECT(vcclAllReduce(s.data(), r.data(), cnt, vcclFloat32, op, c) == vcclInvalidArgument,
         "destroyed op accepted");
  EXPECT_OK(vcclAllReduce(s.data(), r.data(), cnt, vcclFloat32, vcclSum, c));
}

void splitTest(vcclComm_t c, int me, int n) {
  const int color = me % 2;
  vcclComm_t sub = nullptr;
  EXPECT_OK(vcclCommSplit(c, color, me, &sub, nullptr));
  EXPECT(sub != nullptr, "split returned NULL");
  if (sub == nullptr) return;
  int sr = -1, sn = -1;
  EXPECT_OK(vcclCommUserRank(sub, &sr));
  EXPECT_OK(vcclCommCount(sub, &sn));
  EXPECT(sn == (n + (color == 0 ? 1 : 0)) / 2, "split size %d", sn);
  EXPECT(sr == me / 2, "split rank %d", sr);
  std::vector<float> v(64);
  fill(v.data(), vcclFloat32, me, v.size());
  EXPECT_OK(vcclAllReduce(v.data(), v.data(), v.size(), vcclFloat32, vcclSum, sub));
  for (size_t i = 0; i < v.size(); i++) {
    float w = 0;
    for (int p = color; p < n; p += 2) w += val(p, i);
    EXPECT_NEAR(v[i], w, vcclFloat32, "split allreduce", i);
  }
  EXPECT_OK(vcclCommDestroy(sub));
  vcclComm_t sub2 = nullptr;
  EXPECT_OK(vcclCommSplit(c, me == n - 1 ? VCCL_SPLIT_NOCOLOR : 7, 0, &sub2, nullptr));
  if (me == n - 1) EXPECT(sub2 == nullptr, "NOCOLOR rank got a communicator");
  else if (sub2) EXPECT_OK(vcclCommDestroy(sub2));
}

void misc(vcclComm_t c, int me, int n) {
  int ver = 0, dev = -2;
  EXPECT_OK(vcclGetVersion(&ver));
  EXPECT(ver == VCCL_VERSION_CODE, "version");
  EXPECT_OK(vcclCommDevice(c, &dev));
  int cur = -1;
  cudaGetDevice(&cur);
  EXPECT(dev == cur, "device %d != current %d", dev, cur);
  vcclResult_t ae = vcclNumResults;
  EXPECT_OK(vcclCommGetAsyncError(c, &ae));
  EXPECT(ae == vcclSuccess, "async error %d", ae);
  EXPECT_OK(vcclCommFinalize(c));
  // vcclMemAlloc memory is device memory: fill through cudaMemcpy.
  void* mem = nullptr;
  EXPECT_OK(vcclMemAlloc(&mem, 1 << 20));
  vcclMemHandle_t h = nullptr;
  EXPECT_OK(vcclCommRegister(c, mem, 1 << 20, &h));
  std::vector<float> host(256);
  fill(host.data(), vcclFloat32, me, 256);
  cudaMemcpy(mem, host.data(), 1024, cudaMemcpyHostToDevice);
  EXPECT_OK(vcclAllReduce(mem, mem, 256, vcclFloat32, vcclSum, c));
  cudaMemcpy(host.data(), mem, 1024, cudaMemcpyDeviceToHost);
  for (size_t i = 0; i < 256; i++) EXPECT_NEAR(host[i], expect(vcclSum, n, i), vcclFloat32, "memalloc allreduce", i);
  EXPECT_OK(vcclCommDeregister(c, h));
  EXPECT_OK(vcclMemFree(mem));
  EXPECT(vcclMemFree(mem) == vcclInvalidArgument, "double free accepted");
  std::vector<float> b(33);
  if (me == 0) fill(b.data(), vcclFloat32, 0, b.size());
  EXPECT_OK(vcclBcast(b.data(), b.size(), vcclFloat32, 0, c));
  for (size_t i = 0; i < b.size(); i++) EXPECT_NEAR(b[i], val(0, i), vcclFloat32, "bcast", i);
}

void algoAB(vcclComm_t c, int me, int n, size_t cnt) {
  (void)me;
  std::vector<float> s(cnt), r(cnt);
  fill(s.data(), vcclFloat32, me, cnt);
  for (vcclRedOp_t op : {vcclSum, vcclMax}) {
    for (const char* algo : {"ring", "recdouble", "twoshot", "ll", "ll2", "nvls"}) {
      setenv("VCCL_ALLREDUCE_ALGO", algo, 1);
      std::fill(r.begin(), r.end(), -7.0f);
      EXPECT_OK(vcclAllReduce(s.data(), r.data(), cnt, vcclFloat32, op, c));
      for (size_t i = 0; i < cnt; i++) EXPECT_NEAR(r[i], expect(op, n, i), vcclFloat32, algo, i);
    }
    unsetenv("VCCL_ALLREDUCE_ALGO");
  }
  // all-gather A/B (the reference forces ring vs recursive doubling; here
  // pull vs LL), host buffers, each rank's block of cnt / n elements
  const size_t per = cnt / n > 0 ? cnt / n : 1;
  std::vector<float> g(per * n);
  for (const char* algo : {"ring", "recdouble", "pull", "ll"}) {
    setenv("VCCL_ALLGATHER_ALGO", algo, 1);
    std::fill(g.begin(), g.end(), -7.0f);
    EXPECT_OK(vcclAllGather(s.data(), g.data(), per, vcclFloat32, c));
    for (int p = 0; p < n; p++)
      for (size_t i = 0; i < per; i++) EXPECT_NEAR(g[p * per + i], val(p, i), vcclFloat32, algo, i);
  }
  unsetenv("VCCL_ALLGATHER_ALGO");
}

// Device-buffer sweep: every algorithm, sizes up to several staging rounds.
void deviceSweep(vcclComm_t c, int me, int n) {
  const size_t counts[] = {1, 3, 4095, 1 << 14, 300001, 1 << 22, 40u << 20};
  for (vcclDataType_t dt : {vcclFloat32, vcclBfloat16}) {
    const size_t es = vcclTypeSize(dt);
    for (size_t cnt : counts) {
      std::vector<char> h(cnt * es), out(cnt * es);
      fill(h.data(), dt, me, cnt);
      void *ds = nullptr, *dr = nullptr;
      cudaMalloc(&ds, cnt * es);
      cudaMalloc(&dr, cnt * es);
      cudaMemcpy(ds, h.data(), cnt * es, cudaMemcpyHostToDevice);
      for (const char* algo : {"", "ll", "ll2", "twoshot", "nvls"}) {
        if (*algo) setenv("VCCL_ALLREDUCE_ALGO", algo, 1);
        else unsetenv("VCCL_ALLREDUCE_ALGO");
        cudaMemset(dr, 0, cnt * es);
        EXPECT_OK(vcclAllReduceAsync(ds, dr, cnt, dt, vcclSum, c, nullptr));
        cudaDeviceSynchronize();
        cudaMemcpy(out.data(), dr, cnt * es, cudaMemcpyDeviceToHost);
        bool ok = true;
        for (size_t i = 0; i < cnt && ok; i++) {
          if (!near(get(out.data(), dt, i), expect(vcclSum, n, i), dt)) {
            std::fprintf(stderr, "FAIL device allreduce algo=%s dt=%d cnt=%zu i=%zu got %g want %g\n", algo, dt,
                         cnt, i, get(out.data(), dt, i), expect(vcclSum, n, i));
            gFail++;
            ok = false;
          }
        }
      }
      unsetenv("VCCL_ALLREDUCE_ALGO");
      // all-gather / reduce-scatter with device buffers
      const size_t per = cnt / n;
      if (per > 0) {
        void* ag = nullptr;
        cudaMalloc(&ag, per * n * es);
        EXPECT_OK(vcclAllGatherAsync(ds, ag, per, dt, c, nullptr));
        EXPECT_OK(vcclReduceScatterAsync(ds, dr, per, dt, vcclSum, c, nullptr));
        cudaDeviceSynchronize();
        std::vector<char> g(per * n * es), rs(per * es);
        cudaMemcpy(g.data(), ag, g.size(), cudaMemcpyDeviceToHost);
        cudaMemcpy(rs.data(), dr, rs.size(), cudaMemcpyDeviceToHost);
        for (int p = 0; p < n; p++)
          for (size_t i = 0; i < per; i += 97)
            if (!near(get(g.data(), dt, p * per + i), val(p, i), dt)) {
              std::fprintf(stderr, "FAIL device allgather cnt=%zu\n", cnt);
              gFail++;
              break;
            }
        for (size_t i = 0; i < per; i += 97)
          if (!near(get(rs.data(), dt, i), expect(vcclSum, n, me * per + i), dt)) {
            std::fprintf(stderr, "FAIL device reducescatter cnt=%zu i=%zu\n", cnt, i);
            gFail++;
            break;
          }
        cudaFree(ag);
      }
      cudaFree(ds);
      cudaFree(dr);
    }
  }
}

// Messages larger than the staging region: the two-shot and NVLS kernels run
// several rounds with a short last one, the pipelined NVLS kernel reuses its
// slots.  Checked on a stride plus the whole tail.
void multiRound(vcclComm_t c, int me, int n) {
  const size_t cnt = (80u << 20) + 4099;  // > 320 MiB of fp32
  const size_t bytes = cnt * sizeof(float);
  std::vector<float> h(cnt), out(cnt);
  fill(h.data(), vcclFloat32, me, cnt);
  void *ds = nullptr, *dr = nullptr;
  if (cudaMalloc(&ds, bytes) != cudaSuccess || cudaMalloc(&dr, bytes) != cudaSuccess) {
    std::fprintf(stderr, "FAIL multi-round: no device memory\n");
    gFail++;
    return;
  }
  cudaMemcpy(ds, h.data(), bytes, cudaMemcpyHostToDevice);
  for (const char* algo : {"twoshot", "nvls", "nvls_pipe"}) {
    setenv("VCCL_ALLREDUCE_ALGO", algo, 1);
    cudaMemset(dr, 0, bytes);
    EXPECT_OK(vcclAllReduceAsync(ds, dr, cnt, vcclFloat32, vcclSum, c, nullptr));
    cudaDeviceSynchronize();
    cudaMemcpy(out.data(), dr, bytes, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < cnt; i += (i + 70000 < cnt ? 997 : 1)) {
      if (!near(out[i], expect(vcclSum, n, i), vcclFloat32)) {
        std::fprintf(stderr, "FAIL multi-round allreduce algo=%s i=%zu got %g want %g\n", algo, i, out[i],
                     expect(vcclSum, n, i));
        gFail++;
        break;
      }
    }
  }
  unsetenv("VCCL_ALLREDUCE_ALGO");
  cudaFree(ds);
  cudaFree(dr);
}

// Zero-copy collectives on registered windows: all-reduce (point-to-point
// or through the switch, fp32 / bf16, in place, PreMulSum, average, a
// buffer off the 16-byte grid), all-gather into a window, reduce-scatter
// out of one.  Every size is past the LL thresholds so the window kernels
// run.
bool checkDevice(const void* dptr, vcclDataType_t dt, size_t cnt, const char* what,
                 const std::function<float(size_t)>& want) {
  std::vector<char> h(cnt * vcclTypeSize(dt));
  cudaMemcpy(h.data(), dptr, h.size(), cudaMemcpyDeviceToHost);
  for (size_t i = 0; i < cnt; i += (i + 5000 < cnt ? 61 : 1)) {
    if (!near(get(h.data(), dt, i), want(i), dt)) {
      std::fprintf(stderr, "FAIL window %s i=%zu got %g want %g\n", what, i, get(h.data(), dt, i), want(i));
      gFail++;
      return false;
    }
  }
  return true;
}

void windowTest(vcclComm_t c, int me, int n) {
  if (n < 2) return;
  const size_t cnt = (4u << 20) + 5;
  const size_t winBytes = (cnt + 64) * 4 * static_cast<size_t>(n);
  void *a = nullptr, *b = nullptr;
  EXPECT_OK(vcclMemAlloc(&a, winBytes));
  EXPECT_OK(vcclMemAlloc(&b, winBytes));
  vcclWindow_t wa = nullptr, wb = nullptr;
  EXPECT_OK(vcclCommWindowRegister(c, a, winBytes, &wa, 0));
  EXPECT_OK(vcclCommWindowRegister(c, b, winBytes, &wb, 0));
  if (wa == nullptr || wb == nullptr) return;
  auto upload = [&](void* dst, vcclDataType_t dt, size_t count, size_t off) {
    std::vector<char> h(count * vcclTypeSize(dt));
    fill(h.data(), dt, me, count, off);
    cudaMemcpy(dst, h.data(), h.size(), cudaMemcpyHostToDevice);
  };
  char* A = static_cast<char*>(a);
  char* B = static_cast<char*>(b);
  // all-reduce, fp32 and bf16, out of place
  for (vcclDataType_t dt : {vcclFloat32, vcclBfloat16}) {
    upload(A, dt, cnt, 0);
    cudaMemset(B, 0, cnt * vcclTypeSize(dt));
    EXPECT_OK(vcclAllReduce(A, B, cnt, dt, vcclSum, c));
    checkDevice(B, dt, cnt, "allreduce", [&](size_t i) { return expect(vcclSum, n, i); });
  }
  // in place, max
  upload(B, vcclFloat32, cnt, 0);
  EXPECT_OK(vcclAllReduce(B, B, cnt, vcclFloat32, vcclMax, c));
  checkDevice(B, vcclFloat32, cnt, "allreduce in place max", [&](size_t i) { return expect(vcclMax, n, i); });
  // PreMulSum (point-to-point kernel) and average (switch kernel when bound)
  float k = 0.5f;
  vcclRedOp_t pm;
  EXPECT_OK(vcclRedOpCreatePreMulSum(&pm, &k, vcclFloat32, vcclScalarHostImmediate, c));
  upload(A, vcclFloat32, cnt, 0);
  EXPECT_OK(vcclAllReduce(A, B, cnt, vcclFloat32, pm, c));
  checkDevice(B, vcclFloat32, cnt, "allreduce premulsum", [&](size_t i) { return 0.5f * expect(vcclSum, n, i); });
  EXPECT_OK(vcclRedOpDestroy(pm, c));
  EXPECT_OK(vcclAllReduce(A, B, cnt, vcclFloat32, vcclAvg, c));
  checkDevice(B, vcclFloat32, cnt, "allreduce avg", [&](size_t i) { return expect(vcclAvg, n, i); });
  // off the 16-byte grid (element kernels)
  upload(A + 4, vcclFloat32, cnt - 1, 0);
  EXPECT_OK(vcclAllReduce(A + 4, B + 4, cnt - 1, vcclFloat32, vcclSum, c));
  checkDevice(B + 4, vcclFloat32, cnt - 1, "allreduce unaligned", [&](size_t i) { return expect(vcclSum, n, i); });
  // all-gather into window B from a plain buffer
  const size_t per = cnt / n;
  void* local = nullptr;
  cudaMalloc(&local, per * 4);
  upload(local, vcclFloat32, per, 0);
  EXPECT_OK(vcclAllGather(local, B, per, vcclFloat32, c));
  for (int p = 0; p < n; p++) {
    std::vector<float> g(per);
    cudaMemcpy(g.data(), B + p * per * 4, per * 4, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < per; i += 97)
      if (!near(g[i], val(p, i), vcclFloat32)) {
        std::fprintf(stderr, "FAIL window allgather from rank %d i=%zu\n", p, i);
        gFail++;
        break;
      }
  }
  // reduce-scatter out of window A into the plain buffer
  upload(A, vcclFloat32, per * n, 0);
  EXPECT_OK(vcclReduceScatter(A, local, per, vcclFloat32, vcclSum, c));
  checkDevice(local, vcclFloat32, per, "reducescatter", [&](size_t i) { return expect(vcclSum, n, me * per + i); });
  // broadcast from the last rank into window B
  if (me == n - 1) upload(local, vcclFloat32, per, 0);
  EXPECT_OK(vcclBroadcast(local, B, per, vcclFloat32, n - 1, c));
  {
    std::vector<float> g(per), want(per);
    cudaMemcpy(g.data(), B, per * 4, cudaMemcpyDeviceToHost);
    fill(want.data(), vcclFloat32, n - 1, per);
    for (size_t i = 0; i < per; i += 53)
      if (!near(g[i], want[i], vcclFloat32)) {
        std::fprintf(stderr, "FAIL window broadcast i=%zu\n", i);
        gFail++;
        break;
      }
  }
  // all-to-all into window B from window A (equal blocks): block q of rank p
  // lands in rank q's block p
  upload(A, vcclFloat32, per * n, 0);
  EXPECT_OK(vcclAllToAll(A, B, per, vcclFloat32, c));
  for (int p = 0; p < n; p++) {
    std::vector<float> g(per);
    cudaMemcpy(g.data(), B + p * per * 4, per * 4, cudaMemcpyDeviceToHost);
    std::vector<float> want(per * n);
    fill(want.data(), vcclFloat32, p, per * n);
    for (size_t i = 0; i < per; i += 89)
      if (!near(g[i], want[me * per + i], vcclFloat32)) {
        std::fprintf(stderr, "FAIL window alltoall block from rank %d i=%zu\n", p, i);
        gFail++;
        break;
      }
  }
  // all-to-all(v) with uneven blocks into window B: rank p sends
  // 1000 (p + 1) + 7 q elements to rank q, packed in its send buffer
  {
    auto blk = [](int p, int q) { return static_cast<size_t>(1000 * (p + 1) + 7 * q); };
    std::vector<size_t> sc(n), sd(n), rc(n), rd(n);
    size_t so = 0, ro = 0;
    for (int q = 0; q < n; q++) {
      sc[q] = blk(me, q);
      sd[q] = so;
      so += sc[q];
      rc[q] = blk(q, me);
      rd[q] = ro;
      ro += rc[q];
    }
    void* sbuf = nullptr;
    cudaMalloc(&sbuf, so * 4);
    upload(sbuf, vcclFloat32, so, 0);
    EXPECT_OK(vcclAllToAllv(sbuf, sc.data(), sd.data(), B, rc.data(), rd.data(), vcclFloat32, c));
    std::vector<float> g(ro);
    cudaMemcpy(g.data(), B, ro * 4, cudaMemcpyDeviceToHost);
    for (int p = 0; p < n; p++) {
      size_t psd = 0;  // where rank p's block for me starts in its send buffer
      for (int q = 0; q < me; q++) psd += blk(p, q);
      for (size_t i = 0; i < rc[p]; i += 13)
        if (!near(g[rd[p] + i], val(p, psd + i), vcclFloat32)) {
          std::fprintf(stderr, "FAIL window alltoallv from rank %d i=%zu\n", p, i);
          gFail++;
          break;
        }
    }
    cudaFree(sbuf);
  }
  cudaFree(local);
  EXPECT_OK(vcclCommWindowDeregister(c, wa));
  EXPECT_OK(vcclCommWindowDeregister(c, wb));
  EXPECT_OK(vcclMemFree(a));
  EXPECT_OK(vcclMemFree(b));
  // plain cudaMalloc memory: a point-to-point window through CUDA IPC, holding
  // the send buffer and, at the next 4 KiB boundary, the receive buffer
  const size_t ro = (cnt * 4 + 4095) / 4096 * 4096;
  const size_t plainBytes = 2 * ro;
  void* plain = nullptr;
  cudaMalloc(&plain, plainBytes);
  vcclWindow_t wp = nullptr;
  EXPECT_OK(vcclCommWindowRegister(c, plain, plainBytes, &wp, 0));
  if (wp != nullptr) {
    char* P = static_cast<char*>(plain);
    upload(P, vcclFloat32, cnt, 0);
    EXPECT_OK(vcclAllReduce(P, P + ro, cnt, vcclFloat32, vcclSum, c));
    checkDevice(P + ro, vcclFloat32, cnt, "allreduce cudaMalloc window", [&](size_t i) { return expect(vcclSum, n, i); });
    EXPECT_OK(vcclCommWindowDeregister(c, wp));
  }
  cudaFree(plain);
  // host memory: refused on every rank
  std::vector<char> host(1 << 20);
  EXPECT(vcclCommWindowRegister(c, host.data(), host.size(), &wp, 0) == vcclInvalidArgument, "host window");
}

// The pipelined NVLS all-reduce on the device-buffer sweep sizes.
void nvlsPipeSweep(vcclComm_t c, int me, int n) {
  const size_t counts[] = {1, 4095, 300001, 1 << 22, 40u << 20};
  for (size_t cnt : counts) {
    std::vector<float> h(cnt), out(cnt);
    fill(h.data(), vcclFloat32, me, cnt);
    void *ds = nullptr, *dr = nullptr;
    cudaMalloc(&ds, cnt * 4);
    cudaMalloc(&dr, cnt * 4);
    cudaMemcpy(ds, h.data(), cnt * 4, cudaMemcpyHostToDevice);
    setenv("VCCL_ALLREDUCE_ALGO", "nvls_pipe", 1);
    cudaMemset(dr, 0, cnt * 4);
    EXPECT_OK(vcclAllReduceAsync(ds, dr, cnt, vcclFloat32, vcclSum, c, nullptr));
    cudaDeviceSynchronize();
    unsetenv("VCCL_ALLREDUCE_ALGO");
    cudaMemcpy(out.data(), dr, cnt * 4, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < cnt; i++)
      if (!near(out[i], expect(vcclSum, n, i), vcclFloat32)) {
        std::fprintf(stderr, "FAIL nvls_pipe cnt=%zu i=%zu got %g want %g\n", cnt, i, out[i], expect(vcclSum, n, i));
        gFail++;
        break;
      }
    cudaFree(ds);
    cudaFree(dr);
  }
}

// A group whose Send and Recv sit on different streams runs as one kernel
// on the first op's stream; the other stream must still be ordered after
// it: a copy queued on the Recv's stream right after vcclGroupEnd reads the
// received data, not what was there before.
void twoStreamGroup(vcclComm_t c, int me, int n) {
  if (n < 2) return;
  const size_t cnt = 4u << 20;  // 16 MiB of fp32: the kernel outlasts the copy's launch
  const int next = (me + 1) % n, prev = (me + n - 1) % n;
  std::vector<float> h(cnt);
  fill(h.data(), vcclFloat32, me, cnt);
  float *send = nullptr, *recv = nullptr, *host = nullptr;
  cudaMalloc(&send, cnt * 4);
  cudaMalloc(&recv, cnt * 4);
  cudaMallocHost(&host, cnt * 4);
  cudaMemcpy(send, h.data(), cnt * 4, cudaMemcpyHostToDevice);
  cudaMemset(recv, 0, cnt * 4);
  cudaDeviceSynchronize();
  cudaStream_t sa, sb;
  cudaStreamCreateWithFlags(&sa, cudaStreamNonBlocking);
  cudaStreamCreateWithFlags(&sb, cudaStreamNonBlocking);
  EXPECT_OK(vcclGroupStart());
  EXPECT_OK(vcclSendAsync(send, cnt, vcclFloat32, next, c, sa));
  EXPECT_OK(vcclRecvAsync(recv, cnt, vcclFloat32, prev, c, sb));
  EXPECT_OK(vcclGroupEnd());
  cudaMemcpyAsync(host, recv, cnt * 4, cudaMemcpyDeviceToHost, sb);
  cudaStreamSynchronize(sb);
  cudaStreamSynchronize(sa);
  for (size_t i = 0; i < cnt; i += 4099) EXPECT_NEAR(host[i], val(prev, i), vcclFloat32, "two-stream group recv", i);
  EXPECT_NEAR(host[cnt - 1], val(prev, cnt - 1), vcclFloat32, "two-stream group recv", cnt - 1);
  cudaStreamDestroy(sa);
  cudaStreamDestroy(sb);
  cudaFreeHost(host);
  cudaFree(send);
  cudaFree(recv);
}

// Launches of one communicator on two streams run one after the other in
// issue order: the second all-reduce reads the first one's output without
// any synchronisation by the caller.
void twoStreamOrder(vcclComm_t c, int me, int n) {
  const size_t cnt = 4u << 20;
  std::vector<float> h(cnt);
  fill(h.data(), vcclFloat32, me, cnt);
  float *x = nullptr, *y = nullptr, *z = nullptr;
  cudaMalloc(&x, cnt * 4);
  cudaMalloc(&y, cnt * 4);
  cudaMalloc(&z, cnt * 4);
  cudaMemcpy(x, h.data(), cnt * 4, cudaMemcpyHostToDevice);
  cudaMemset(y, 0, cnt * 4);
  cudaMemset(z, 0, cnt * 4);
  cudaDeviceSynchronize();
  cudaStream_t sa, sb;
  cudaStreamCreateWithFlags(&sa, cudaStreamNonBlocking);
  cudaStreamCreateWithFlags(&sb, cudaStreamNonBlocking);
  EXPECT_OK(vcclAllReduceAsync(x, y, cnt, vcclFloat32, vcclSum, c, sa));
  EXPECT_OK(vcclAllReduceAsync(y, z, cnt, vcclFloat32, vcclSum, c, sb));
  cudaStreamSynchronize(sb);
  cudaStreamSynchronize(sa);
  cudaMemcpy(h.data(), z, cnt * 4, cudaMemcpyDeviceToHost);
  for (size_t i = 0; i < cnt; i += 4099)
    EXPECT_NEAR(h[i], n * expect(vcclSum, n, i), vcclFloat32, "two-stream order", i);
  cudaStreamDestroy(sa);
  cudaStreamDestroy(sb);
  cudaFree(x);
  cudaFree(y);
  cudaFree(z);
}

// Paths added after the main matrix was validated on B200 run in their own
// invocation (`test_collectives N --extended`), so a failure there cannot
// hide the main matrix's result.
bool gExtended = false;

int rankMain(int me, int n, const vcclUniqueId& id, bool full) {
  cudaSetDevice(me);
  vcclComm_t c = nullptr;
  EXPECT_OK(vcclCommInitRank(&c, n, id, me));
  if (c == nullptr) return 1;
  if (gExtended) {
    nvlsPipeSweep(c, me, n);
    multiRound(c, me, n);
    windowTest(c, me, n);
    twoStreamGroup(c, me, n);
    twoStreamOrder(c, me, n);
    if (std::getenv("VCCL_GUARDS") != nullptr && n > 1) {
      unsigned long long bad = 0;
      EXPECT_OK(vcclxCheckGuards(c, &bad));
      EXPECT(bad == 0, "kernels wrote past their regions");
    }
    EXPECT_OK(vcclCommDestroy(c));
    if (gFail) std::fprintf(stderr, "rank %d/%d: %d failures (extended)\n", me, n, gFail);
    return gFail ? 1 : 0;
  }
  int r = -1, cnt = -1;
  EXPECT_OK(vcclCommUserRank(c, &r));
  EXPECT_OK(vcclCommCount(c, &cnt));
  EXPECT(r == me && cnt == n, "rank/count");
  const size_t sizes[] = {1, 7, 1024, (1 << 16) + 3};
  const vcclDataType_t dts[] = {vcclFloat32, vcclFloat16, vcclBfloat16, vcclInt32, vcclFloat64};
  for (size_t s : sizes) {
    for (vcclDataType_t dt : dts) {
      allGather(c, me, n, dt, s);
      reduceScatter(c, me, n, dt, vcclSum, s);
      allReduce(c, me, n, dt, vcclSum, s);
      allReduce(c, me, n, dt, vcclMax, s);
      allReduce(c, me, n, dt, vcclMin, s);
    }
    allReduce(c, me, n, vcclFloat32, vcclAvg, s);
    reduceAll(c, me, n, vcclFloat32, vcclSum, s);
    reduceAll(c, me, n, vcclFloat32, vcclMax, s);
    broadcastAll(c, me, n, s);
    sendRecvPairs(c, me, n, s);
    groupNeighbours(c, me, n, s);
  }
  reduceAll(c, me, n, vcclFloat16, vcclSum, 511);
  reduceAll(c, me, n, vcclFloat32, vcclAvg, 257);
  allReduce(c, me, n, vcclFloat32, vcclProd, 1000);
  gatherScatter(c, me, n, 1000);
  allToAll(c, me, n, 333);
  preMulSum(c, me, n, 512);
  splitTest(c, me, n);
  misc(c, me, n);
  algoAB(c, me, n, 1000);
  algoAB(c, me, n, 70000);
  if (full) deviceSweep(c, me, n);
  EXPECT_OK(vcclCommDestroy(c));
  if (gFail) std::fprintf(stderr, "rank %d/%d: %d failures\n", me, n, gFail);
  return gFail ? 1 : 0;
}

int forkRanks(int n, bool full) {
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
  std::vector<pid_t> pids;
  for (int r = 0; r < n; r++) {
    pid_t p = fork();
    if (p == 0) _exit(rankMain(r, n, id, full));
    pids.push_back(p);
  }
  int bad = 0;
  for (pid_t p : pids) {
    int st = 0;
    waitpid(p, &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) bad++;
  }
  std::printf("nranks=%d: %s\n", n, bad ? "FAIL" : "OK");
  std::fflush(stdout);
  return bad ? 1 : 0;
}

// One rank leaves between steps (no kernel of its in flight); survivors'
// next collective must time out on the device, report an error, and latch
// the communicator so the following call fails fast.
int killRank(int me, int n, const vcclUniqueId& id, int victim) {
  cudaSetDevice(me);
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, n, id, me) != vcclSuccess) return 2;
  std::vector<float> buf(4096, 1.0f);
  if (vcclAllReduce(buf.data(), buf.data(), buf.size(), vcclFloat32, vcclSum, c) != vcclSuccess) return 3;
  if (me == victim) _exit(0);
  usleep(200 * 1000);
  vcclResult_t r1 = vcclAllReduce(buf.data(), buf.data(), buf.size(), vcclFloat32, vcclSum, c);
  vcclResult_t r2 = vcclAllReduce(buf.data(), buf.data(), buf.size(), vcclFloat32, vcclSum, c);
  vcclResult_t ae = vcclSuccess;
  vcclCommGetAsyncError(c, &ae);
  vcclCommDestroy(c);
  const bool ok = r1 != vcclSuccess && r2 == vcclInvalidUsage && ae != vcclSuccess;
  if (!ok) std::fprintf(stderr, "kill survivor %d: r1=%d r2=%d async=%d\n", me, r1, r2, ae);
  return ok ? 0 : 1;
}

int runKill(int n) {
  setenv("VCCL_TIMEOUT", "3", 1);
  setenv("VCCL_NVLS_ENABLE", "0", 1);
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
  const int victim = 1;
  auto t0 = std::chrono::steady_clock::now();
  std::vector<pid_t> pids;
  for (int r = 0; r < n; r++) {
    pid_t p = fork();
    if (p == 0) _exit(killRank(r, n, id, victim));
    pids.push_back(p);
  }
  int bad = 0;
  for (size_t i = 0; i < pids.size(); i++) {
    int st = 0;
    waitpid(pids[i], &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) bad++;
  }
  const long secs = std::chrono::duration_cast<std::chrono::seconds>(std::chrono::steady_clock::now() - t0).count();
  if (secs > 60) bad++;
  unsetenv("VCCL_TIMEOUT");
  unsetenv("VCCL_NVLS_ENABLE");
  std::printf("kill-a-rank (nranks=%d, %lds): %s\n", n, secs, bad ? "FAIL" : "OK");
  std::fflush(stdout);
  return bad ? 1 : 0;
}

// vcclCommAbort from another thread while a kernel waits: rank 1 never
// launches the collective (its failure is injected on the host), so rank 0's
// kernel waits for it; a thread of rank 0 aborts after 300 ms, the kernel
// sees the host-mapped abort word and returns well before the (30 s)
// timeout, and the communicator is latched.  NVLS off, as for kill-a-rank.
int abortRank(int me, int n, const vcclUniqueId& id) {
  cudaSetDevice(me);
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, n, id, me) != vcclSuccess) return 2;
  const size_t cnt = 1u << 20;
  float* d = nullptr;
  cudaMalloc(&d, cnt * 4);
  cudaMemset(d, 0, cnt * 4);
  int rc = 0;
  if (me == 0) {
    cudaStream_t st;
    cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    auto t0 = std::chrono::steady_clock::now();
    std::thread aborter([c]() {
      std::this_thread::sleep_for(std::chrono::milliseconds(300));
      vcclCommAbort(c);
    });
    const vcclResult_t r0 = vcclAllReduceAsync(d, d, cnt, vcclFloat32, vcclSum, c, st);
    cudaStreamSynchronize(st);
    aborter.join();
    const double secs =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    const vcclResult_t r1 = vcclAllReduce(d, d, cnt, vcclFloat32, vcclSum, c);
    vcclResult_t ae = vcclSuccess;
    vcclCommGetAsyncError(c, &ae);
    const bool ok = r0 == vcclSuccess && r1 == vcclInvalidUsage && ae != vcclSuccess && secs < 10.0;
    if (!ok) std::fprintf(stderr, "abort rank 0: launch=%d next=%d async=%d after %.1f s\n", r0, r1, ae, secs);
    rc = ok ? 0 : 1;
    cudaStreamDestroy(st);
  } else {
    std::this_thread::sleep_for(std::chrono::milliseconds(2000));  // skips the collective
  }
  cudaFree(d);
  vcclCommDestroy(c);
  return rc;
}

int runAbort(int n) {
  setenv("VCCL_TIMEOUT", "30", 1);
  setenv("VCCL_NVLS_ENABLE", "0", 1);
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
  std::vector<pid_t> pids;
  for (int r = 0; r < n; r++) {
    pid_t p = fork();
    if (p == 0) _exit(abortRank(r, n, id));
    pids.push_back(p);
  }
  int bad = 0;
  for (pid_t p : pids) {
    int st = 0;
    waitpid(p, &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) bad++;
  }
  unsetenv("VCCL_TIMEOUT");
  unsetenv("VCCL_NVLS_ENABLE");
  std::printf("abort while a kernel waits (nranks=%d): %s\n", n, bad ? "FAIL" : "OK");
  std::fflush(stdout);
  return bad ? 1 : 0;
}

int initAll(int ndev) {
  std::vector<vcclComm_t> comms(ndev, nullptr);
  if (vcclCommInitAll(comms.data(), ndev, nullptr) != vcclSuccess) {
    std::printf("init-all: FAIL (init)\n");
    return 1;
  }
  std::vector<float*> bufs(ndev);
  for (int d = 0; d < ndev; d++) {
    cudaSetDevice(d);
    cudaMalloc(&bufs[d], 128 * sizeof(float));
    std::vector<float> h(128);
    fill(h.data(), vcclFloat32, d, 128);
    cudaMemcpy(bufs[d], h.data(), 512, cudaMemcpyHostToDevice);
  }
  int bad = 0;
  if (vcclGroupStart() != vcclSuccess) bad++;
  for (int d = 0; d < ndev; d++)
    if (vcclAllReduce(bufs[d], bufs[d], 128, vcclFloat32, vcclSum, comms[d]) != vcclSuccess) bad++;
  if (vcclGroupEnd() != vcclSuccess) bad++;
  for (int d = 0; d < ndev; d++) {
    cudaSetDevice(d);
    std::vector<float> h(128);
    cudaMemcpy(h.data(), bufs[d], 512, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < 128; i++)
      if (h[i] != expect(vcclSum, ndev, i)) bad++;
    cudaFree(bufs[d]);
    vcclCommDestroy(comms[d]);
  }
  std::printf("init-all group allreduce (%d devices): %s\n", ndev, bad ? "FAIL" : "OK");
  return bad ? 1 : 0;
}

// Windows between ranks of one process (vcclCommInitAll): a cudaMalloc
// buffer per device, registered and all-reduced from one thread per rank
// (registration is collective, so every rank must be inside the call).
int initAllWindow(int ndev) {
  std::vector<vcclComm_t> comms(ndev, nullptr);
  if (vcclCommInitAll(comms.data(), ndev, nullptr) != vcclSuccess) {
    std::printf("init-all window: FAIL (init)\n");
    return 1;
  }
  const size_t cnt = (2u << 20) + 3;
  std::vector<int> bad(ndev, 0);
  std::vector<std::thread> th;
  for (int d = 0; d < ndev; d++)
    th.emplace_back([&, d]() {
      cudaSetDevice(d);
      char* buf = nullptr;
      const size_t ro = (cnt * 4 + 4095) / 4096 * 4096;
      cudaMalloc(&buf, ro + cnt * 4);
      std::vector<float> h(cnt);
      fill(h.data(), vcclFloat32, d, cnt);
      cudaMemcpy(buf, h.data(), cnt * 4, cudaMemcpyHostToDevice);
      vcclWindow_t w = nullptr;
      if (vcclCommWindowRegister(comms[d], buf, ro + cnt * 4, &w, 0) != vcclSuccess) {
        bad[d]++;
      } else {
        if (vcclAllReduce(buf, buf + ro, cnt, vcclFloat32, vcclSum, comms[d]) != vcclSuccess) bad[d]++;
        cudaMemcpy(h.data(), buf + ro, cnt * 4, cudaMemcpyDeviceToHost);
        for (size_t i = 0; i < cnt; i += 31)
          if (!near(h[i], expect(vcclSum, ndev, i), vcclFloat32)) {
            bad[d]++;
            break;
          }
        if (vcclCommWindowDeregister(comms[d], w) != vcclSuccess) bad[d]++;
      }
      cudaFree(buf);
    });
  for (auto& t : th) t.join();
  int total = 0;
  for (int d = 0; d < ndev; d++) {
    total += bad[d];
    vcclCommDestroy(comms[d]);
  }
  std::printf("init-all window allreduce (%d devices): %s\n", ndev, total ? "FAIL" : "OK");
  return total ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
  // Count GPUs in a child so the parent never initialises CUDA before fork.
  int ngpu = 0;
  {
    int fds[2];
    if (pipe(fds) != 0) return 1;
    pid_t p = fork();
    if (p == 0) {
      int n = 0;
      if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
      if (write(fds[1], &n, sizeof(n)) != sizeof(n)) _exit(1);
      _exit(0);
    }
    if (read(fds[0], &ngpu, sizeof(ngpu)) != sizeof(ngpu)) ngpu = 0;
    waitpid(p, nullptr, 0);
    close(fds[0]);
    close(fds[1]);
  }
  int maxRanks = argc > 1 ? std::atoi(argv[1]) : ngpu;
  if (maxRanks > ngpu) maxRanks = ngpu;
  if (maxRanks < 1) {
    std::printf("no GPU visible: skipped\n");
    return 77;
  }
  int fails = 0;
  if (argc > 2 && std::strcmp(argv[2], "--extended") == 0) {
    gExtended = true;
    if (maxRanks >= 2) fails += forkRanks(2, true);
    if (maxRanks > 2) fails += forkRanks(maxRanks, true);
    if (maxRanks == 1) fails += forkRanks(1, true);
    if (maxRanks >= 2) fails += runAbort(2);
    if (maxRanks >= 2) {
      pid_t p = fork();
      if (p == 0) _exit(initAllWindow(std::min(maxRanks, 4)));
      int st = 0;
      waitpid(p, &st, 0);
      if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) fails++;
    }
    if (fails == 0) std::printf("all tests passed\n");
    return fails ? 1 : 0;
  }
  if (maxRanks >= 2) fails += runKill(std::min(maxRanks, 4));
  for (int n = 1; n <= maxRanks; n++) {
    if (n > 2 && n != maxRanks && n != 3 && n != 5) continue;  // 1,2,3,5 and the largest
    fails += forkRanks(n, n == maxRanks);
  }
  if (maxRanks >= 2) {
    pid_t p = fork();
    if (p == 0) _exit(initAll(std::min(maxRanks, 3)));
    int st = 0;
    waitpid(p, &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) fails++;
  }
  if (fails == 0) std::printf("all tests passed\n");
  return fails ? 1 : 0;
}
