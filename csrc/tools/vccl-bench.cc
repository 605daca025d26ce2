// SPDX-License-Identifier: Apache-2.0
// vccl-bench: bandwidth / latency sweep of the collectives on GPUs.
//
// Same command line and busbw conventions as the reference bench (reference:
// bench/vccl_bench.cc:30-40 options, :147-152 busbw factors, :154-236 run
// loop): --launch N forks N local ranks, -b/-e/-f size sweep, --iters,
// --warmup, --dtype, --check, --op allreduce|allgather|reducescatter|
// broadcast|alltoall.  Differences: buffers are device memory, time is
// measured with CUDA events on the launching stream and reported as the
// maximum over ranks, --algo forces an all-reduce algorithm, --graph times a
// captured loop, and --window puts both buffers in registered windows
// (vcclMemAlloc + vcclCommWindowRegister: the zero-copy kernels).  --host
// (also taken without a GPU or with VCCL_NO_DEVICE=1) runs communicators
// without a device on host buffers over the host data plane, timed by the
// host clock like the reference's bench (maximum over ranks).
// Multi-process launch: VCCL_RANK / VCCL_NRANKS and VCCL_COMM_ID or
// VCCL_ID_FILE, as in the reference.
#include <cuda_runtime.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "vccl.h"

namespace {

struct Opts {
  std::string op = "allreduce";
  size_t minBytes = 1024, maxBytes = 64u << 20;
  double factor = 2.0;
  int iters = 20, warmup = 3, launch = 0;
  bool check = false;
  bool graph = false;
  bool window = false;
  bool host = false;
  vcclDataType_t dt = vcclFloat32;
  std::string algo;
};

size_t parseSize(const char* s) {
  char* e = nullptr;
  double v = std::strtod(s, &e);
  if (e && (*e == 'K' || *e == 'k')) v *= 1024;
  if (e && (*e == 'M' || *e == 'm')) v *= 1024 * 1024;
  if (e && (*e == 'G' || *e == 'g')) v *= 1024.0 * 1024 * 1024;
  return static_cast<size_t>(v);
}

double busFactor(const std::string& op, int n) {
  if (op == "allreduce") return 2.0 * (n - 1) / n;
  if (op == "allgather" || op == "reducescatter" || op == "alltoall") return static_cast<double>(n - 1) / n;
  return 1.0;
}

[[noreturn]] void usage() {
  std::fprintf(stderr,
               "usage: vccl-bench [--launch N] [--op allreduce|allgather|reducescatter|broadcast|alltoall]\n"
               "                  [-b min] [-e max] [-f factor] [--iters N] [--warmup N]\n"
               "                  [--dtype f32|f16|bf16|f64] [--algo ll|twoshot|nvls|nvls_pipe] [--check]\n"
               "                  [--graph] [--window] [--host]\n");
  std::exit(2);
}

__global__ void fillPattern(float* p, size_t n, int rank) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    p[i] = static_cast<float>((rank + i) % 8);
}

// Copies results back for the checks (host buffers: a plain copy).
void fetch(bool host, float* dst, const float* src, size_t cnt) {
  if (host) {
    std::memcpy(dst, src, cnt * 4);
  } else {
    cudaMemcpy(dst, src, cnt * 4, cudaMemcpyDeviceToHost);
  }
}

int checkF32(const Opts& o, vcclComm_t c, int rank, int n, float* s, float* r, size_t bytes, bool host) {
  const size_t cnt = bytes / 4, per = cnt / n;
  if (host) {
    for (size_t i = 0; i < cnt; i++) s[i] = static_cast<float>((rank + i) % 8);
  } else {
    fillPattern<<<256, 256>>>(s, cnt, rank);
    cudaDeviceSynchronize();
  }
  std::vector<float> h;
  size_t bad = 0;
  if (o.op == "allreduce") {
    vcclAllReduce(s, r, cnt, vcclFloat32, vcclSum, c);
    h.resize(cnt);
    fetch(host, h.data(), r, cnt);
    for (size_t i = 0; i < cnt; i++) {
      float w = 0;
      for (int p = 0; p < n; p++) w += static_cast<float>((p + i) % 8);
      if (h[i] != w) bad++;
    }
  } else if (o.op == "allgather") {
    vcclAllGather(s, r, per, vcclFloat32, c);
    h.resize(per * n);
    fetch(host, h.data(), r, per * n);
    for (int p = 0; p < n; p++)
      for (size_t i = 0; i < per; i++)
        if (h[p * per + i] != static_cast<float>((p + i) % 8)) bad++;
  } else if (o.op == "reducescatter") {
    vcclReduceScatter(s, r, per, vcclFloat32, vcclSum, c);
    h.resize(per);
    fetch(host, h.data(), r, per);
    for (size_t i = 0; i < per; i++) {
      float w = 0;
      for (int p = 0; p < n; p++) w += static_cast<float>((p + rank * per + i) % 8);
      if (h[i] != w) bad++;
    }
  } else {
    return 0;
  }
  if (bad) {
    std::fprintf(stderr, "rank %d: %s check FAILED (%zu mismatches)\n", rank, o.op.c_str(), bad);
    return 1;
  }
  std::printf("# rank %d: %s correctness check passed\n", rank, o.op.c_str());
  return 0;
}

// The sweep on host buffers (communicator without a device), host clock.
int runHostRank(const Opts& o, int rank, int n, const vcclUniqueId& id) {
  setenv("VCCL_NO_DEVICE", "1", 1);
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, n, id, rank) != vcclSuccess) {
    std::fprintf(stderr, "rank %d: init failed: %s\n", rank, vcclGetLastError(nullptr));
    return 1;
  }
  const size_t es = vcclTypeSize(o.dt);
  const size_t cap = o.maxBytes + 4096;
  std::vector<float> sv(cap / 4 + 1, 0.0f), rv(cap / 4 + 1, 0.0f);
  char* s = reinterpret_cast<char*>(sv.data());
  char* r = reinterpret_cast<char*>(rv.data());
  if (o.check && checkF32(o, c, rank, n, sv.data(), rv.data(), o.maxBytes, true)) return 1;
  if (rank == 0) {
    std::printf("# op=%s dtype_bytes=%zu nranks=%d iters=%d warmup=%d (host buffers, host data plane; "
                "host clock, max over ranks)\n",
                o.op.c_str(), es, n, o.iters, o.warmup);
    std::printf("%14s %12s %12s %12s\n", "bytes", "time(us)", "algbw(GB/s)", "busbw(GB/s)");
  }
  for (size_t bytes = o.minBytes; bytes <= o.maxBytes;
       bytes = std::max(bytes + 1, static_cast<size_t>(bytes * o.factor))) {
    const size_t cnt = bytes / es, per = cnt / n;
    if (cnt == 0) continue;
    if ((o.op == "allgather" || o.op == "reducescatter" || o.op == "alltoall") && per == 0) continue;
    auto once = [&]() -> vcclResult_t {
      if (o.op == "allreduce") return vcclAllReduce(s, r, cnt, o.dt, vcclSum, c);
      if (o.op == "allgather") return vcclAllGather(s, r, per, o.dt, c);
      if (o.op == "reducescatter") return vcclReduceScatter(s, r, per, o.dt, vcclSum, c);
      if (o.op == "broadcast") return vcclBroadcast(s, r, cnt, o.dt, 0, c);
      if (o.op == "alltoall") return vcclAllToAll(s, r, per, o.dt, c);
      return vcclInvalidArgument;
    };
    for (int i = 0; i < o.warmup; i++)
      if (once() != vcclSuccess) return 1;
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < o.iters; i++)
      if (once() != vcclSuccess) return 1;
    float us = std::chrono::duration<float, std::micro>(std::chrono::steady_clock::now() - t0).count() / o.iters;
    if (vcclAllReduce(&us, &us, 1, vcclFloat32, vcclMax, c) != vcclSuccess) return 1;
    if (rank == 0) {
      const double eff = (o.op == "allgather" || o.op == "reducescatter" || o.op == "alltoall")
                             ? static_cast<double>(per * n * es)
                             : static_cast<double>(cnt * es);
      const double algbw = eff / (us * 1e3);
      std::printf("%14zu %12.2f %12.2f %12.2f\n", static_cast<size_t>(eff), us, algbw, algbw * busFactor(o.op, n));
    }
  }
  vcclCommDestroy(c);
  return 0;
}

int runRank(const Opts& o, int rank, int n, const vcclUniqueId& id) {
  setvbuf(stdout, nullptr, _IOLBF, 0);
  const char* nd = std::getenv("VCCL_NO_DEVICE");
  if (o.host || (nd && std::atoi(nd) != 0)) return runHostRank(o, rank, n, id);
  int ngpu = 0;
  if (cudaGetDeviceCount(&ngpu) != cudaSuccess || ngpu < 1) {
    cudaGetLastError();
    if (rank == 0) std::printf("# no CUDA device: host buffers over the host data plane\n");
    return runHostRank(o, rank, n, id);
  }
  cudaSetDevice(rank % ngpu);
  if (!o.algo.empty()) setenv("VCCL_ALLREDUCE_ALGO", o.algo.c_str(), 1);
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, n, id, rank) != vcclSuccess) {
    std::fprintf(stderr, "rank %d: init failed: %s\n", rank, vcclGetLastError(nullptr));
    return 1;
  }
  const size_t es = vcclTypeSize(o.dt);
  void *s = nullptr, *r = nullptr;
  size_t cap = o.maxBytes + 4096;
  if (o.op == "allgather") cap = o.maxBytes + 4096;
  vcclWindow_t ws = nullptr, wr = nullptr;
  if (o.window) {
    if (vcclMemAlloc(&s, cap) != vcclSuccess || vcclMemAlloc(&r, cap) != vcclSuccess ||
        vcclCommWindowRegister(c, s, cap, &ws, 0) != vcclSuccess ||
        vcclCommWindowRegister(c, r, cap, &wr, 0) != vcclSuccess) {
      std::fprintf(stderr, "rank %d: window set-up failed: %s\n", rank, vcclGetLastError(c));
      return 1;
    }
  } else {
    cudaMalloc(&s, cap);
    cudaMalloc(&r, cap);
  }
  cudaMemset(s, 0, cap);
  if (o.check && checkF32(o, c, rank, n, static_cast<float*>(s), static_cast<float*>(r), o.maxBytes, false)) return 1;
  cudaStream_t st;
  cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  float* tMax = nullptr;
  cudaMalloc(&tMax, sizeof(float));
  if (rank == 0) {
    std::printf("# op=%s dtype_bytes=%zu nranks=%d iters=%d warmup=%d (device time, max over ranks)\n",
                o.op.c_str(), es, n, o.iters, o.warmup);
    std::printf("%14s %12s %12s %12s\n", "bytes", "time(us)", "algbw(GB/s)", "busbw(GB/s)");
  }
  for (size_t bytes = o.minBytes; bytes <= o.maxBytes;
       bytes = std::max(bytes + 1, static_cast<size_t>(bytes * o.factor))) {
    size_t cnt = bytes / es;
    size_t per = cnt / n;
    if (cnt == 0) continue;
    if ((o.op == "allgather" || o.op == "reducescatter" || o.op == "alltoall") && per == 0) continue;
    auto once = [&]() -> vcclResult_t {
      if (o.op == "allreduce") return vcclAllReduceAsync(s, r, cnt, o.dt, vcclSum, c, st);
      if (o.op == "allgather") return vcclAllGatherAsync(s, r, per, o.dt, c, st);
      if (o.op == "reducescatter") return vcclReduceScatterAsync(s, r, per, o.dt, vcclSum, c, st);
      if (o.op == "broadcast") return vcclBroadcastAsync(s, r, cnt, o.dt, 0, c, st);
      if (o.op == "alltoall") return vcclAllToAllAsync(s, r, per, o.dt, c, st);
      return vcclInvalidArgument;
    };
    for (int i = 0; i < o.warmup; i++)
      if (once() != vcclSuccess) return 1;
    cudaStreamSynchronize(st);
    cudaGraphExec_t exec = nullptr;
    if (o.graph) {
      // Device time without host launch overhead: replay a captured loop.
      cudaGraph_t g = nullptr;
      cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
      for (int i = 0; i < o.iters; i++) once();
      cudaStreamEndCapture(st, &g);
      if (g == nullptr || cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) {
        std::fprintf(stderr, "graph capture failed\n");
        return 1;
      }
      cudaGraphDestroy(g);
      cudaGraphLaunch(exec, st);  // warm the graph
      cudaStreamSynchronize(st);
    }
    cudaEventRecord(e0, st);
    if (exec) {
      cudaGraphLaunch(exec, st);
    } else {
      for (int i = 0; i < o.iters; i++)
        if (once() != vcclSuccess) return 1;
    }
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    if (exec) cudaGraphExecDestroy(exec);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    float us = ms * 1000.0f / o.iters;
    cudaMemcpy(tMax, &us, sizeof(float), cudaMemcpyHostToDevice);
    vcclAllReduce(tMax, tMax, 1, vcclFloat32, vcclMax, c);
    cudaMemcpy(&us, tMax, sizeof(float), cudaMemcpyDeviceToHost);
    vcclResult_t ae = vcclSuccess;
    vcclCommGetAsyncError(c, &ae);
    if (ae != vcclSuccess) {
      std::fprintf(stderr, "rank %d: async error %d: %s\n", rank, ae, vcclGetLastError(c));
      return 1;
    }
    if (rank == 0) {
      const double eff = (o.op == "allgather" || o.op == "reducescatter" || o.op == "alltoall")
                             ? static_cast<double>(per * n * es)
                             : static_cast<double>(cnt * es);
      const double algbw = eff / (us * 1e3);
      std::printf("%14zu %12.2f %12.2f %12.2f\n", static_cast<size_t>(eff), us, algbw, algbw * busFactor(o.op, n));
    }
  }
  if (o.window) {
    vcclCommWindowDeregister(c, ws);
    vcclCommWindowDeregister(c, wr);
    vcclMemFree(s);
    vcclMemFree(r);
  } else {
    cudaFree(s);
    cudaFree(r);
  }
  cudaFree(tMax);
  vcclCommDestroy(c);
  return 0;
}

bool writeId(const char* path, const vcclUniqueId& id) {
  std::string tmp = std::string(path) + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "w");
  if (!f) return false;
  for (int i = 0; i < VCCL_UNIQUE_ID_BYTES; i++) std::fprintf(f, "%02x", static_cast<unsigned char>(id.internal[i]));
  std::fprintf(f, "\n");
  std::fclose(f);
  return std::rename(tmp.c_str(), path) == 0;
}

bool readId(const char* path, vcclUniqueId* id) {
  for (int t = 0; t < 1200; t++) {
    FILE* f = std::fopen(path, "r");
    if (f) {
      char buf[2 * VCCL_UNIQUE_ID_BYTES + 4] = {0};
      bool ok = std::fgets(buf, sizeof(buf), f) && std::strlen(buf) >= 2 * VCCL_UNIQUE_ID_BYTES;
      std::fclose(f);
      if (ok) {
        for (int i = 0; i < VCCL_UNIQUE_ID_BYTES; i++) {
          unsigned v = 0;
          std::sscanf(buf + 2 * i, "%02x", &v);
          id->internal[i] = static_cast<char>(v);
        }
        return true;
      }
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(100));
  }
  return false;
}

}  // namespace

int main(int argc, char** argv) {
  Opts o;
  for (int i = 1; i < argc; i++) {
    std::string a = argv[i];
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) usage();
      return argv[++i];
    };
    if (a == "--op") o.op = next();
    else if (a == "-b") o.minBytes = parseSize(next());
    else if (a == "-e") o.maxBytes = parseSize(next());
    else if (a == "-f") o.factor = std::atof(next());
    else if (a == "--iters") o.iters = std::atoi(next());
    else if (a == "--warmup") o.warmup = std::atoi(next());
    else if (a == "--launch") o.launch = std::atoi(next());
    else if (a == "--check") o.check = true;
    else if (a == "--graph") o.graph = true;
    else if (a == "--window") o.window = true;
    else if (a == "--host") o.host = true;
    else if (a == "--algo") o.algo = next();
    else if (a == "--dtype") {
      std::string d = next();
      if (d == "f32") o.dt = vcclFloat32;
      else if (d == "f16") o.dt = vcclFloat16;
      else if (d == "bf16") o.dt = vcclBfloat16;
      else if (d == "f64") o.dt = vcclFloat64;
      else usage();
    } else usage();
  }
  if (o.factor <= 1.0) o.factor = 2.0;
  if (o.launch > 0) {
    setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
    vcclUniqueId id;
    if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
    std::vector<pid_t> pids;
    for (int r = 0; r < o.launch; r++) {
      pid_t p = fork();
      if (p == 0) _exit(runRank(o, r, o.launch, id));
      pids.push_back(p);
    }
    int bad = 0;
    for (pid_t p : pids) {
      int st = 0;
      waitpid(p, &st, 0);
      if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) bad++;
    }
    return bad ? 1 : 0;
  }
  const char* re = std::getenv("VCCL_RANK");
  const char* ne = std::getenv("VCCL_NRANKS");
  const char* idFile = std::getenv("VCCL_ID_FILE");
  const char* commId = std::getenv("VCCL_COMM_ID");
  if (!re || !ne || (!idFile && !commId)) {
    std::fprintf(stderr, "set VCCL_RANK, VCCL_NRANKS and VCCL_COMM_ID or VCCL_ID_FILE, or use --launch N\n");
    return 2;
  }
  const int rank = std::atoi(re), n = std::atoi(ne);
  vcclUniqueId id;
  if (commId || rank == 0) {
    if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
    if (!commId && !writeId(idFile, id)) return 1;
  } else if (!readId(idFile, &id)) {
    std::fprintf(stderr, "timed out waiting for %s\n", idFile);
    return 1;
  }
  return runRank(o, rank, n, id);
}
