// SPDX-License-Identifier: Apache-2.0
// Collective entry points, group semantics and host-buffer staging.
//
// Argument rules follow the reference (reference: src/core/collectives.cc:
// 63-98 and :756-905): a dead communicator returns vcclInvalidUsage, avg and
// PreMulSum are float-only, PreMulSum resolves to sum plus a pre-scale of the
// caller's own contribution, send/recv reject peer == self, root-only
// buffers may be NULL elsewhere, count tables of AllToAllv are copied so they
// outlive a group.  Group semantics follow reference: src/core/group.cc:
// 25-125: thread-local nesting, per-communicator issue order, consecutive
// point-to-point operations progressed together (here: in one kernel).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <thread>
#include <vector>

#include "common/env.h"
#include "common/log.h"
#include "common/trace.h"
#include "runtime/comm.h"
#include "runtime/cudrv.h"
#include "runtime/launch.h"

namespace vccl {

LaunchCtx launchCtxFor(const DeviceState& ds, cudaStream_t s) {
  LaunchCtx lc;
  lc.dc = ds.dc;
  lc.stream = s;
  lc.nblocks = ds.nblocks;
  lc.nvls = ds.nvls;
  lc.llMax = ds.llMaxBytes;
  lc.llAgMax = ds.llAgMaxBytes;
  lc.llBlocks = ds.llBlocks;
  lc.nvlsPieces = ds.nvlsPieces;
  return lc;
}

namespace {

enum class Kind { AllReduce, Reduce, AllGather, ReduceScatter, Broadcast, Gather, Scatter, AllToAllv, Send, Recv };

struct HostOp {
  Kind kind;
  vcclComm_t comm;
  const char* send = nullptr;
  char* recv = nullptr;
  size_t count = 0;
  vcclDataType_t dt = vcclFloat32;
  int redKind = dev::kSum;
  bool avg = false;
  bool premul = false;
  double scalar = 1.0;
  int root = -1;
  int peer = -1;
  std::vector<size_t> sc, sd, rc, rd;
  cudaStream_t stream = nullptr;
  bool sync = true;     // host-blocking semantics
  bool staged = false;  // host pointers allowed (staged through device memory)
  // Windows the registration cache picked for this call on every rank (null:
  // only application windows are looked up).
  const Window* winSend = nullptr;
  const Window* winRecv = nullptr;
};

thread_local int tDepth = 0;
thread_local std::vector<HostOp> tQueue;

bool isFloat(vcclDataType_t dt) {
  return dt == vcclFloat16 || dt == vcclFloat32 || dt == vcclFloat64 || dt == vcclBfloat16 ||
         dt == vcclFloat8e4m3 || dt == vcclFloat8e5m2;
}

vcclResult_t usable(vcclComm_t comm) {
  if (comm == nullptr) return vcclInvalidArgument;
  if (comm->aborted.load()) {
    VERR("communicator is aborted; destroy it and create a new one");
    return vcclInvalidUsage;
  }
  vcclResult_t st = comm->pollDeviceStatus();
  if (st != vcclSuccess) {
    comm->noteError(st);
    return vcclInvalidUsage;
  }
  return vcclSuccess;
}

vcclResult_t resolveOp(vcclComm_t comm, vcclDataType_t dt, vcclRedOp_t op, HostOp* h) {
  if (static_cast<int>(op) < 0) return vcclInvalidArgument;
  if (op >= vcclNumOps) {
    double s = 1.0;
    if (!comm->premulScalar(op, &s) || !isFloat(dt)) return vcclInvalidArgument;
    h->premul = true;
    h->scalar = s;
    h->redKind = dev::kSum;
    return vcclSuccess;
  }
  switch (op) {
    case vcclSum: h->redKind = dev::kSum; break;
    case vcclProd: h->redKind = dev::kProd; break;
    case vcclMax: h->redKind = dev::kMax; break;
    case vcclMin: h->redKind = dev::kMin; break;
    case vcclAvg:
      if (!isFloat(dt)) return vcclInvalidArgument;
      h->redKind = dev::kSum;
      h->avg = true;
      break;
    default: return vcclInvalidArgument;
  }
  return vcclSuccess;
}

// ---- pointer classification and staging ------------------------------------
enum class PtrKind { Null, Host, Device, OtherDevice };

PtrKind classify(const void* p, int device) {
  if (p == nullptr) return PtrKind::Null;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return PtrKind::Host;
  }
  if (at.type == cudaMemoryTypeDevice) return at.device == device ? PtrKind::Device : PtrKind::OtherDevice;
  if (at.type == cudaMemoryTypeManaged) return PtrKind::Device;
  return PtrKind::Host;
}

struct StageRange {
  char* host;
  size_t bytes;
  char* devp;
  bool copyBack;
};

struct Staging {
  std::vector<StageRange> ranges;
  // Map a host pointer range to device memory; inputs are copied in.
  vcclResult_t map(cudaStream_t s, const char* host, size_t bytes, bool input, bool output, char** out) {
    if (bytes == 0) {
      *out = const_cast<char*>(host);
      return vcclSuccess;
    }
    for (StageRange& r : ranges) {
      if (host >= r.host && host + bytes <= r.host + r.bytes) {
        *out = r.devp + (host - r.host);
        r.copyBack |= output;
        return vcclSuccess;
      }
    }
    void* d = nullptr;
    if (cudaMallocAsync(&d, bytes, s) != cudaSuccess) {
      VERR("staging allocation of %zu bytes failed", bytes);
      return vcclSystemError;
    }
    if (input && cudaMemcpyAsync(d, host, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) return vcclSystemError;
    ranges.push_back({const_cast<char*>(host), bytes, static_cast<char*>(d), output});
    *out = static_cast<char*>(d);
    return vcclSuccess;
  }
  vcclResult_t finish(cudaStream_t s) {
    vcclResult_t res = vcclSuccess;
    for (StageRange& r : ranges) {
      if (r.copyBack && cudaMemcpyAsync(r.host, r.devp, r.bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        res = vcclSystemError;
      cudaFreeAsync(r.devp, s);
    }
    ranges.clear();
    return res;
  }
};

struct Extents {
  size_t in = 0, out = 0;
  bool needIn = true, needOut = true;
};

Extents extentsOf(const HostOp& h) {
  const size_t es = vcclTypeSize(h.dt);
  const size_t n = static_cast<size_t>(h.comm->nranks);
  const int me = h.comm->rank;
  Extents e;
  switch (h.kind) {
    case Kind::AllReduce: e.in = e.out = h.count * es; break;
    case Kind::Reduce: e.in = h.count * es; e.out = h.count * es; e.needOut = me == h.root; break;
    case Kind::AllGather: e.in = h.count * es; e.out = n * h.count * es; break;
    case Kind::ReduceScatter: e.in = n * h.count * es; e.out = h.count * es; break;
    case Kind::Broadcast: e.in = h.count * es; e.out = h.count * es; e.needIn = me == h.root; break;
    case Kind::Gather: e.in = h.count * es; e.out = n * h.count * es; e.needOut = me == h.root; break;
    case Kind::Scatter: e.in = n * h.count * es; e.out = h.count * es; e.needIn = me == h.root; break;
    case Kind::AllToAllv:
      for (size_t p = 0; p < n; p++) {
        e.in = std::max(e.in, (h.sd[p] + h.sc[p]) * es);
        e.out = std::max(e.out, (h.rd[p] + h.rc[p]) * es);
      }
      break;
    case Kind::Send: e.in = h.count * es; e.needOut = false; break;
    case Kind::Recv: e.out = h.count * es; e.needIn = false; break;
  }
  return e;
}

// Replace host pointers by staged device pointers (blocking calls) or
// reject them (stream-ordered calls).
vcclResult_t prepareBuffers(HostOp& h, Staging& st) {
  const int device = h.comm->device();
  Extents e = extentsOf(h);
  const bool recvUsed = e.needOut && h.recv != nullptr;
  const bool sendUsed = e.needIn && h.send != nullptr;
  PtrKind rk = recvUsed ? classify(h.recv, device) : PtrKind::Null;
  PtrKind sk = sendUsed ? classify(h.send, device) : PtrKind::Null;
  if (rk == PtrKind::OtherDevice || sk == PtrKind::OtherDevice) {
    VERR("buffer belongs to another CUDA device than the communicator's (%d)", device);
    return vcclInvalidArgument;
  }
  if ((rk == PtrKind::Host || sk == PtrKind::Host) && !h.staged) {
    VERR("stream-ordered collectives take device pointers; got a host pointer");
    return vcclInvalidArgument;
  }
  // In-place forms: the send range lies inside the receive range.
  const bool aliased = sendUsed && recvUsed && h.send >= h.recv && h.send + e.in <= h.recv + e.out;
  if (rk == PtrKind::Host) {
    char* d = nullptr;
    VTRY(st.map(h.stream, h.recv, e.out, aliased, true, &d));
    if (aliased) {
      h.send = d + (h.send - h.recv);
      sk = PtrKind::Device;
    }
    h.recv = d;
  }
  if (sk == PtrKind::Host) {
    char* d = nullptr;
    VTRY(st.map(h.stream, h.send, e.in, true, false, &d));
    h.send = d;
  }
  return vcclSuccess;
}

LaunchCtx launchCtx(vcclComm_t comm, cudaStream_t s) { return launchCtxFor(*comm->dev, s); }

vcclResult_t cudaToVccl(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return vcclSuccess;
  VERR("%s: %s", what, cudaGetErrorString(e));
  return e == cudaErrorInvalidValue ? vcclInvalidArgument : vcclUnhandledError;
}

ArAlgo pickAllReduce(const HostOp& h, size_t bytes) {
  const DeviceState& ds = *h.comm->dev;
  // Read on every call (tests and sweeps switch it between calls); no
  // allocation unless it is set.
  const char* forced = std::getenv("VCCL_ALLREDUCE_ALGO");
  std::string force = forced != nullptr ? forced : "";
  if (force.empty() && !ds.tuning.empty()) force = tunedAlgorithm(ds.tuning, "allreduce", h.comm->nranks, bytes);
  const bool llOk = bytes <= dev::kLLMaxBytes &&
                    ((reinterpret_cast<uintptr_t>(h.send) | reinterpret_cast<uintptr_t>(h.recv)) & 7u) == 0;
  const bool nvlsOk = ds.nvls && nvlsSupports(h.dt, h.redKind);
  const int n = h.comm->nranks;
  const bool aligned = ((reinterpret_cast<uintptr_t>(h.send) | reinterpret_cast<uintptr_t>(h.recv)) & 7u) == 0;
  const bool ll2Ok = aligned && ((bytes + 7) / 8 + n - 1) / n * 8 <= dev::kLLMaxBytes;
  if (force == "ll" || force == "oneshot" || force == "recdouble") {
    if (llOk) return ArAlgo::LL;
  } else if (force == "ll2") {
    if (ll2Ok) return ArAlgo::LL2;
  } else if (force == "nvls") {
    if (nvlsOk) return ArAlgo::Nvls;
  } else if (force == "nvls_pipe") {
    if (nvlsOk) return ArAlgo::NvlsPipe;
  } else if (force == "twoshot" || force == "ring") {
    return ArAlgo::TwoShot;
  }
  if (llOk && bytes <= ds.llMaxBytes) return ArAlgo::LL;
  if (ll2Ok && bytes <= ds.ll2MaxBytes) return ArAlgo::LL2;
  // Per GPU, NVLS moves (1 + 1/n) S each way against 2 (n-1)/n S for the
  // two-shot: it only wins from four ranks on.
  if (nvlsOk && h.comm->nranks >= ds.nvlsMinRanks && bytes >= ds.nvlsMinBytes)
    return ds.nvlsPipeMin != 0 && bytes >= ds.nvlsPipeMin ? ArAlgo::NvlsPipe : ArAlgo::Nvls;
  return ArAlgo::TwoShot;
}

// Point-to-point plan builder.
struct PlanBuilder {
  dev::P2pPlan plan;
  std::map<std::pair<int, int>, int> maxCh;  // (peer, kind) -> channels
  bool anyCopy = false;
  PlanBuilder() { memset(&plan, 0, sizeof(plan)); }
  vcclResult_t add(int kind, int peer, char* dst, const char* src, size_t bytes) {
    if (plan.nops >= dev::kMaxP2pOps) {
      VERR("too many point-to-point operations in one group (max %d)", dev::kMaxP2pOps);
      return vcclInvalidUsage;
    }
    plan.ops[plan.nops++] = {dst, src, bytes, peer, kind};
    if (kind == dev::kP2pCopy) {
      anyCopy = true;
    } else {
      int& m = maxCh[{peer, kind}];
      m = std::max(m, dev::p2pChannels(bytes));
    }
    return vcclSuccess;
  }
  vcclResult_t finalize() {
    plan.nwork = 0;
    for (auto& kv : maxCh) {
      for (int ch = 0; ch < kv.second; ch++) {
        if (plan.nwork >= dev::kMaxP2pWork) return vcclInvalidUsage;
        plan.work[plan.nwork++] = {static_cast<int16_t>(kv.first.first), static_cast<int8_t>(kv.first.second),
                                   static_cast<int8_t>(ch)};
      }
    }
    if (anyCopy)
      for (int ch = 0; ch < dev::kMaxChannels; ch++) {
        if (plan.nwork >= dev::kMaxP2pWork) return vcclInvalidUsage;
        plan.work[plan.nwork++] = {-1, static_cast<int8_t>(dev::kP2pCopy), static_cast<int8_t>(ch)};
      }
    return vcclSuccess;
  }
};

// Translate a root-based or pairwise collective into point-to-point work.
vcclResult_t addP2pWork(const HostOp& h, PlanBuilder& pb) {
  const size_t es = vcclTypeSize(h.dt);
  const int n = h.comm->nranks, me = h.comm->rank;
  const size_t chunk = h.count * es;
  switch (h.kind) {
    case Kind::Send: return pb.add(dev::kP2pSend, h.peer, nullptr, h.send, chunk);
    case Kind::Recv: return pb.add(dev::kP2pRecv, h.peer, h.recv, nullptr, chunk);
    case Kind::Gather:
      if (me != h.root) return pb.add(dev::kP2pSend, h.root, nullptr, h.send, chunk);
      for (int p = 0; p < n; p++) {
        if (p == me) {
          if (h.recv + p * chunk != h.send) VTRY(pb.add(dev::kP2pCopy, p, h.recv + p * chunk, h.send, chunk));
        } else {
          VTRY(pb.add(dev::kP2pRecv, p, h.recv + p * chunk, nullptr, chunk));
        }
      }
      return vcclSuccess;
    case Kind::Scatter:
      if (me != h.root) return pb.add(dev::kP2pRecv, h.root, h.recv, nullptr, chunk);
      for (int p = 0; p < n; p++) {
        if (p == me) {
          if (h.send + p * chunk != h.recv) VTRY(pb.add(dev::kP2pCopy, p, h.recv, h.send + p * chunk, chunk));
        } else {
          VTRY(pb.add(dev::kP2pSend, p, nullptr, h.send + p * chunk, chunk));
        }
      }
      return vcclSuccess;
    case Kind::AllToAllv:
      for (int s = 0; s < n; s++) {
        const int to = (me + s) % n;
        if (to == me) {
          if (h.sc[me] > 0 && h.recv + h.rd[me] * es != h.send + h.sd[me] * es)
            VTRY(pb.add(dev::kP2pCopy, me, h.recv + h.rd[me] * es, h.send + h.sd[me] * es, h.sc[me] * es));
          continue;
        }
        VTRY(pb.add(dev::kP2pSend, to, nullptr, h.send + h.sd[to] * es, h.sc[to] * es));
        VTRY(pb.add(dev::kP2pRecv, to, h.recv + h.rd[to] * es, nullptr, h.rc[to] * es));
      }
      return vcclSuccess;
    default: return vcclInternalError;
  }
}

bool isP2pKind(Kind k) { return k == Kind::Send || k == Kind::Recv; }
bool usesP2pKernel(Kind k) {
  return k == Kind::Send || k == Kind::Recv || k == Kind::Gather || k == Kind::Scatter || k == Kind::AllToAllv;
}

// The algorithm the latest launch on this thread chose (read back for the
// call profile, VCCL_PROF=1).
thread_local const char* tAlgo = nullptr;

void chose(const char* op, const char* algo, int nranks, size_t bytes) {
  tAlgo = algo;
  noteAlgorithm(op, algo, nranks, bytes);
}

const char* opName(Kind k) {
  switch (k) {
    case Kind::AllReduce: return "all-reduce";
    case Kind::Reduce: return "reduce";
    case Kind::AllGather: return "all-gather";
    case Kind::ReduceScatter: return "reduce-scatter";
    case Kind::Broadcast: return "broadcast";
    case Kind::Gather: return "gather";
    case Kind::Scatter: return "scatter";
    case Kind::AllToAllv: return "all-to-all(v)";
    case Kind::Send: return "send";
    case Kind::Recv: return "recv";
  }
  return "?";
}

// Bytes a call names (count x type size; all-to-all(v): this rank's sends).
size_t callBytes(const HostOp& h) {
  const size_t es = vcclTypeSize(h.dt);
  if (h.kind != Kind::AllToAllv) return h.count * es;
  size_t t = 0;
  for (size_t c : h.sc) t += c * es;
  return t;
}

// Launch one non-p2p collective (device pointers by now).
const char* kindName(Kind k) {
  switch (k) {
    case Kind::AllReduce: return "vccl AllReduce";
    case Kind::Reduce: return "vccl Reduce";
    case Kind::AllGather: return "vccl AllGather";
    case Kind::ReduceScatter: return "vccl ReduceScatter";
    case Kind::Broadcast: return "vccl Broadcast";
    case Kind::Gather: return "vccl Gather";
    case Kind::Scatter: return "vccl Scatter";
    case Kind::AllToAllv: return "vccl AllToAllv";
    case Kind::Send: return "vccl Send";
    case Kind::Recv: return "vccl Recv";
  }
  return "vccl";
}

const char* algoName(ArAlgo a) {
  switch (a) {
    case ArAlgo::LL: return "one-shot LL";
    case ArAlgo::LL2: return "two-hop LL";
    case ArAlgo::Nvls: return "NVLS multimem";
    case ArAlgo::NvlsPipe: return "NVLS multimem, pipelined";
    case ArAlgo::TwoShot: return "two-shot";
  }
  return "?";
}

// Zero-copy path for buffers in registered windows (runtime/window.cc):
// all-reduce with both buffers in windows, all-gather with the receive
// buffer in one, reduce-scatter with the send buffer in one.  Messages the
// LL protocol handles stay on it.  Every rank decides alike: the windows,
// offsets and counts agree across ranks by the window rule (the kernels
// check it).
bool windowCollective(const HostOp& h, const LaunchCtx& lc, vcclResult_t* out) {
  vcclComm_t comm = h.comm;
  const DeviceState& ds = *comm->dev;
  if (!ds.windowsEnabled) return false;
  const size_t es = vcclTypeSize(h.dt);
  const int n = comm->nranks, me = comm->rank;
  const size_t bytes = h.count * es;
  dev::WinArgs w{};
  w.count = h.count;
  w.premul = h.premul ? 1 : 0;
  w.avg = h.avg ? 1 : 0;
  w.scalar = h.scalar;
  auto bindSend = [&](const Window* win) {
    w.sendOff = static_cast<uint64_t>(h.send - win->base);
    for (int q = 0; q < n; q++) w.send[q] = win->peer[q] + w.sendOff;
    w.mcSend = win->mc ? win->mc + w.sendOff : nullptr;
  };
  auto bindRecv = [&](const Window* win) {
    w.recvOff = static_cast<uint64_t>(h.recv - win->base);
    for (int q = 0; q < n; q++) w.recv[q] = win->peer[q] + w.recvOff;
    w.mcRecv = win->mc ? win->mc + w.recvOff : nullptr;
  };
  const bool switchRanks = n >= ds.windowNvlsMinRanks;
  cudaError_t e = cudaSuccess;
  switch (h.kind) {
    case Kind::AllReduce: {
      if (bytes <= ds.llMaxBytes) return false;
      const Window* ws = h.winSend ? h.winSend : comm->findWindow(h.send, bytes);
      const Window* wr = h.winRecv ? h.winRecv : comm->findWindow(h.recv, bytes);
      if (ws == nullptr || wr == nullptr) return false;
      bindSend(ws);
      bindRecv(wr);
      bool sw = switchRanks && w.mcSend != nullptr && w.mcRecv != nullptr;
      e = launchAllReduceWindow(lc, h.dt, h.redKind, w, sw);
      if (e == cudaErrorInvalidValue && sw) {  // datatype, operation or alignment the switch cannot take
        cudaGetLastError();
        sw = false;
        e = launchAllReduceWindow(lc, h.dt, h.redKind, w, false);
      }
      chose("all-reduce", sw ? "window NVLS" : "window two-shot", n, bytes);
      *out = cudaToVccl(e, "window all-reduce launch");
      return true;
    }
    case Kind::AllGather: {
      if (bytes <= lc.llAgMax) return false;
      const Window* wr = h.winRecv ? h.winRecv : comm->findWindow(h.recv, bytes * n);
      if (wr == nullptr) return false;
      bindRecv(wr);
      w.send[me] = h.send;  // the send buffer is read locally only
      w.count = bytes;
      chose("all-gather", w.mcRecv ? "window multimem push" : "window push", n, bytes);
      *out = cudaToVccl(launchAllGatherWindow(lc, w), "window all-gather launch");
      return true;
    }
    case Kind::Broadcast: {
      if (bytes <= lc.llMax) return false;
      const Window* wr = h.winRecv ? h.winRecv : comm->findWindow(h.recv, bytes);
      if (wr == nullptr) return false;
      bindRecv(wr);
      w.send[me] = h.send;  // read on the root only
      w.count = bytes;
      chose("broadcast", w.mcRecv ? "window multimem" : "window push", n, bytes);
      *out = cudaToVccl(launchBroadcastWindow(lc, w, h.root), "window broadcast launch");
      return true;
    }
    case Kind::ReduceScatter: {
      if (bytes <= lc.llMax) return false;
      const Window* ws = h.winSend ? h.winSend : comm->findWindow(h.send, bytes * n);
      if (ws == nullptr) return false;
      bindSend(ws);
      w.recv[me] = h.recv;  // written locally only
      chose("reduce-scatter", switchRanks && w.mcSend ? "window NVLS" : "window pull", n, bytes);
      *out = cudaToVccl(launchReduceScatterWindow(lc, h.dt, h.redKind, w, switchRanks), "window reduce-scatter launch");
      return true;
    }
    default:
      return false;
  }
}

// Registration cache (VCCL_REG_CACHE=1): windows over the buffers of a large
// all-reduce / all-gather / reduce-scatter / broadcast on plain device
// memory, reused across calls (runtime/regcache.h).  Whether a call consults
// the cache depends only on its kind and size, which agree across ranks, so
// every rank takes part in the cache's allgather for the same calls.
// `eligible`: no buffer of this rank was a staged host range.
vcclResult_t cacheWindowsFor(HostOp& h, bool eligible) {
  vcclComm_t comm = h.comm;
  const size_t n = static_cast<size_t>(comm->nranks);
  const size_t bytes = h.count * vcclTypeSize(h.dt);
  const void* ptrs[kRegMaxBuffers] = {nullptr, nullptr};
  size_t sizes[kRegMaxBuffers] = {0, 0};
  int nbuf = 1;
  switch (h.kind) {
    case Kind::AllReduce:
      // Where the staged NVLS all-reduce runs (NVLS, enough ranks), it moves
      // less data per GPU than the point-to-point kernel of a cached window
      // (cudaMalloc windows have no multicast binding): keep it.
      if (comm->dev->nvls && comm->nranks >= comm->dev->nvlsMinRanks) return vcclSuccess;
      ptrs[0] = h.send;
      sizes[0] = bytes;
      if (h.recv != h.send) {
        ptrs[1] = h.recv;
        sizes[1] = bytes;
        nbuf = 2;
      }
      break;
    case Kind::AllGather: ptrs[0] = h.recv; sizes[0] = bytes * n; break;
    case Kind::ReduceScatter: ptrs[0] = h.send; sizes[0] = bytes * n; break;
    case Kind::Broadcast: ptrs[0] = h.recv; sizes[0] = bytes; break;
    default: return vcclSuccess;
  }
  if (sizes[0] < comm->dev->regCacheMin) return vcclSuccess;
  const Window* w[kRegMaxBuffers] = {nullptr, nullptr};
  VTRY(regCacheWindows(comm, h.stream, ptrs, sizes, nbuf, eligible, w));
  switch (h.kind) {
    case Kind::AllReduce:
      h.winSend = w[0];
      h.winRecv = nbuf == 2 ? w[1] : w[0];
      if (h.winSend == nullptr || h.winRecv == nullptr) h.winSend = h.winRecv = nullptr;
      break;
    case Kind::ReduceScatter: h.winSend = w[0]; break;
    default: h.winRecv = w[0]; break;
  }
  return vcclSuccess;
}

// Zero-copy all-to-all(v) with the receive buffer in a registered window:
// every rank writes its blocks straight into the peers' receive buffers, at
// the displacements each receiver publishes on the device.  The window, or
// null when this does not apply (the slot-ring kernel runs).  Decided on the
// caller's pointers, before any staging: a receive buffer in a window is
// device memory.  Every rank takes the same path: windows are registered,
// and the receive buffer lies in one on every rank (the window rule).
const Window* windowForAllToAll(const HostOp& h) {
  vcclComm_t comm = h.comm;
  const int n = comm->nranks;
  if (!comm->dev || !comm->dev->windowsEnabled || n == 1 || comm->windows.empty()) return nullptr;
  size_t extent = 0;
  for (int q = 0; q < n; q++) extent = std::max(extent, h.rd[q] + h.rc[q]);
  const size_t es = vcclTypeSize(h.dt);
  return extent == 0 ? nullptr : comm->findWindow(h.recv, extent * es);
}

vcclResult_t windowAllToAll(const HostOp& h, const Window* wr) {
  vcclComm_t comm = h.comm;
  const int n = comm->nranks, me = comm->rank;
  const size_t es = vcclTypeSize(h.dt);
  dev::WinArgs w{};
  w.recvOff = static_cast<uint64_t>(h.recv - wr->base);
  for (int q = 0; q < n; q++) w.recv[q] = wr->peer[q] + w.recvOff;
  w.send[me] = h.send;
  dev::A2aTable t{};
  size_t total = 0;
  for (int q = 0; q < n; q++) {
    t.sc[q] = h.sc[q];
    t.sd[q] = h.sd[q];
    t.rc[q] = h.rc[q];
    t.rd[q] = h.rd[q];
    total += h.sc[q] * es;
  }
  w.count = 0;  // counts differ per rank; the table check covers them
  chose("all-to-all(v)", "window push", n, total);
  return cudaToVccl(launchAllToAllvWindow(launchCtx(comm, h.stream), w, t, static_cast<int>(es)),
                    "window all-to-all(v) launch");
}

vcclResult_t launchColl(const HostOp& h) {
  vcclComm_t comm = h.comm;
  const size_t es = vcclTypeSize(h.dt);
  const int n = comm->nranks;
  cudaStream_t s = h.stream;
  if (h.count == 0) return vcclSuccess;
  TraceRange trace(kindName(h.kind));
  if (n == 1) {
    double scale = h.premul ? h.scalar : 1.0;
    switch (h.kind) {
      case Kind::AllReduce: case Kind::Reduce: case Kind::ReduceScatter: case Kind::AllGather:
        return cudaToVccl(launchScaleCopy(s, h.dt, h.recv, h.send, h.count, scale), "single-rank copy");
      case Kind::Broadcast:
        return cudaToVccl(launchScaleCopy(s, h.dt, h.recv, h.send, h.count, 1.0), "single-rank copy");
      default: return vcclInternalError;
    }
  }
  LaunchCtx lc = launchCtx(comm, s);
  vcclResult_t winResult = vcclSuccess;
  if (!comm->windows.empty() && windowCollective(h, lc, &winResult)) return winResult;
  dev::CollArgs a{h.send, h.recv, h.count, -1, h.premul ? 1 : 0, h.avg ? 1 : 0, h.scalar};
  switch (h.kind) {
    case Kind::AllReduce: {
      ArAlgo algo = pickAllReduce(h, h.count * es);
      chose("all-reduce", algoName(algo), n, h.count * es);
      cudaError_t e = launchAllReduce(lc, algo, h.dt, h.redKind, a);
      if (e == cudaErrorInvalidValue && algo != ArAlgo::TwoShot) {
        cudaGetLastError();
        e = launchAllReduce(lc, ArAlgo::TwoShot, h.dt, h.redKind, a);
      }
      return cudaToVccl(e, "all-reduce launch");
    }
    case Kind::Reduce:
      a.root = h.root;
      return cudaToVccl(launchAllReduce(lc, ArAlgo::TwoShot, h.dt, h.redKind, a), "reduce launch");
    case Kind::ReduceScatter:
      chose("reduce-scatter", h.count * es <= lc.llMax ? "LL" : "push", n, h.count * es);
      return cudaToVccl(launchReduceScatter(lc, h.dt, h.redKind, a), "reduce-scatter launch");
    case Kind::AllGather: {
      // VCCL_ALLGATHER_ALGO forces the algorithm (read per call, as the
      // all-reduce override is): ll / oneshot / recdouble take the LL kernel
      // whenever the message allows it, pull / ring the pull kernel.
      LaunchCtx agc = lc;
      const char* forced = std::getenv("VCCL_ALLGATHER_ALGO");
      if (forced != nullptr) {
        const std::string f = forced;
        if (f == "ll" || f == "oneshot" || f == "recdouble") agc.llAgMax = dev::kLLMaxBytes;
        else if (f == "pull" || f == "ring") agc.llAgMax = 0;
      }
      chose("all-gather", h.count * es <= agc.llAgMax ? "LL" : "pull", n, h.count * es);
      return cudaToVccl(launchAllGather(agc, h.send, h.recv, h.count * es), "all-gather launch");
    }
    case Kind::Broadcast: {
      const size_t bytes = h.count * es;
      std::string force = envStr("VCCL_BROADCAST_ALGO", "");
      if (force.empty() && !comm->dev->tuning.empty()) force = tunedAlgorithm(comm->dev->tuning, "broadcast", n, bytes);
      // The root sends S through the switch instead of (n-1) S to the peers.
      bool nv = lc.nvls && (force == "nvls" || (force.empty() && n >= 3 && bytes >= (256u << 10)));
      chose("broadcast", bytes <= lc.llMax ? "LL" : nv ? "NVLS multimem" : "pull", n, bytes);
      return cudaToVccl(launchBroadcast(lc, h.send, h.recv, bytes, h.root, nv), "broadcast launch");
    }
    default: return vcclInternalError;
  }
}

// Host-only path for single-rank communicators without a device.
vcclResult_t runHostSingle(const HostOp& h) {
  const size_t es = vcclTypeSize(h.dt);
  const size_t bytes = h.count * es;
  switch (h.kind) {
    case Kind::AllReduce: case Kind::Reduce: case Kind::ReduceScatter: case Kind::AllGather:
    case Kind::Broadcast: case Kind::Gather: case Kind::Scatter:
      if (h.recv && h.send && h.recv != h.send && bytes) memmove(h.recv, h.send, bytes);
      break;
    case Kind::AllToAllv:
      if (h.sc[0]) memmove(h.recv + h.rd[0] * es, h.send + h.sd[0] * es, h.sc[0] * es);
      break;
    default: return vcclInvalidUsage;
  }
  if (h.premul && h.kind != Kind::Broadcast) {
    if (h.dt == vcclFloat32) {
      float* p = reinterpret_cast<float*>(h.recv);
      for (size_t i = 0; i < h.count; i++) p[i] = static_cast<float>(p[i] * h.scalar);
    } else if (h.dt == vcclFloat64) {
      double* p = reinterpret_cast<double*>(h.recv);
      for (size_t i = 0; i < h.count; i++) p[i] *= h.scalar;
    } else {
      VERR("PreMulSum on a device-less communicator supports f32/f64 only");
      return vcclInvalidUsage;
    }
  }
  return vcclSuccess;
}

struct PendingSync {
  vcclComm_t comm;
  cudaStream_t stream;
};

// Launch a communicator's ops in order.  Streams that must be waited on for
// blocking semantics are appended to `waits`.
// One operation of a device-less communicator with several ranks, on the
// host data plane (host memory only).
vcclResult_t runHostPlane(HostPlane& hp, const HostOp& h) {
  const size_t es = vcclTypeSize(h.dt);
  const HostRed r{h.dt, h.redKind, h.avg, h.premul, h.scalar};
  switch (h.kind) {
    case Kind::AllReduce: return hp.allReduce(h.send, h.recv, h.count, r);
    case Kind::Reduce: return hp.reduce(h.send, h.recv, h.count, r, h.root);
    case Kind::ReduceScatter: return hp.reduceScatter(h.send, h.recv, h.count, r);
    case Kind::AllGather: return hp.allGather(h.send, h.recv, h.count * es);
    case Kind::Broadcast: return hp.broadcast(h.send, h.recv, h.count * es, h.root);
    case Kind::Gather: return hp.gather(h.send, h.recv, h.count * es, h.root);
    case Kind::Scatter: return hp.scatter(h.send, h.recv, h.count * es, h.root);
    case Kind::AllToAllv: {
      const size_t n = h.sc.size();
      std::vector<size_t> sc(n), sd(n), rc(n), rd(n);
      for (size_t p = 0; p < n; p++) {
        sc[p] = h.sc[p] * es;
        sd[p] = h.sd[p] * es;
        rc[p] = h.rc[p] * es;
        rd[p] = h.rd[p] * es;
      }
      return hp.allToAllv(h.send, sc.data(), sd.data(), h.recv, rc.data(), rd.data());
    }
    default: return vcclInternalError;
  }
}

// Device-less communicators: one rank copies locally; several ranks move
// host memory over the host data plane (made on the first data call, which
// every rank reaches in the same order).
vcclResult_t launchHostOps(vcclComm_t comm, std::vector<HostOp>& ops) {
  if (comm->nranks == 1) {
    for (const HostOp& h : ops) {
      VTRY(runHostSingle(h));
      comm->noteCall(opName(h.kind), "host", callBytes(h));
    }
    return vcclSuccess;
  }
  for (const HostOp& h : ops) {
    if (!h.staged) {
      VERR("a communicator without a device takes host buffers through the blocking calls only");
      return vcclInvalidUsage;
    }
    // Without a CUDA driver every pointer is host memory; with one (a GPU
    // host running VCCL_NO_DEVICE=1), device pointers are refused.
    if (driverApi() == nullptr) continue;
    for (const char* p : {static_cast<const char*>(h.send), static_cast<const char*>(h.recv)}) {
      if (p != nullptr && classify(p, -1) != PtrKind::Host) {
        VERR("a communicator without a device moves host memory only; got a device pointer");
        return vcclInvalidArgument;
      }
    }
  }
  HostPlane* hp = nullptr;
  {
    std::lock_guard<std::mutex> g(comm->hostPlaneMu);
    hp = comm->hostPlane.get();
  }
  if (hp == nullptr) {
    std::unique_ptr<HostPlane> made;
    VTRY(HostPlane::create(comm->bootstrap.get(), &made));
    std::lock_guard<std::mutex> g(comm->hostPlaneMu);
    comm->hostPlane = std::move(made);
    hp = comm->hostPlane.get();
  }
  size_t i = 0;
  while (i < ops.size()) {
    const HostOp& h = ops[i];
    if (isP2pKind(h.kind)) {
      // A run of sends and receives progresses together (group semantics).
      std::vector<HostXfer> xs;
      size_t j = i;
      for (; j < ops.size() && isP2pKind(ops[j].kind); j++) {
        const HostOp& o = ops[j];
        const size_t bytes = o.count * vcclTypeSize(o.dt);
        if (o.peer == comm->rank) return vcclInvalidArgument;
        xs.push_back({o.kind == Kind::Send, o.peer,
                      o.kind == Kind::Send ? const_cast<char*>(o.send) : o.recv, bytes});
        comm->noteCall(opName(o.kind), "host TCP mesh", bytes);
      }
      VTRY(hp->run(xs));
      i = j;
      continue;
    }
    VTRY(runHostPlane(*hp, h));
    comm->noteCall(opName(h.kind), hp->path(), callBytes(h));
    i++;
  }
  return vcclSuccess;
}

vcclResult_t launchOps(vcclComm_t comm, std::vector<HostOp>& ops, std::vector<PendingSync>* waits) {
  if (!comm->dev) return launchHostOps(comm, ops);
  cudaSetDevice(comm->dev->device);
  size_t i = 0;
  while (i < ops.size()) {
    HostOp& h = ops[i];
    Staging st;
    const Window* a2aWin = h.kind == Kind::AllToAllv ? windowForAllToAll(h) : nullptr;
    if (a2aWin != nullptr) {
      OrderedLaunch ord(comm->dev.get(), h.stream);
      VTRY(prepareBuffers(h, st));  // a host send buffer is staged; the receive buffer is device memory
      VTRY(windowAllToAll(h, a2aWin));
      VTRY(st.finish(h.stream));
      comm->noteCall(opName(h.kind), "window push", callBytes(h));
      if (h.sync) waits->push_back({comm, h.stream});
      i++;
      continue;
    }
    if (usesP2pKernel(h.kind)) {
      if (comm->nranks == 1) {
        // Only self copies exist (gather/scatter/all-to-all on one rank).
        VTRY(prepareBuffers(h, st));
        const size_t es = vcclTypeSize(h.dt);
        if (h.kind == Kind::AllToAllv) {
          if (h.sc[0] && h.recv + h.rd[0] * es != h.send + h.sd[0] * es)
            VTRY(cudaToVccl(cudaMemcpyAsync(h.recv + h.rd[0] * es, h.send + h.sd[0] * es, h.sc[0] * es,
                                            cudaMemcpyDefault, h.stream), "copy"));
        } else if (h.count && h.recv != h.send) {
          VTRY(cudaToVccl(cudaMemcpyAsync(h.recv, h.send, h.count * es, cudaMemcpyDefault, h.stream), "copy"));
        }
        VTRY(st.finish(h.stream));
        comm->noteCall(opName(h.kind), "local copy", callBytes(h));
        if (h.sync) waits->push_back({comm, h.stream});
        i++;
        continue;
      }
      // A maximal run of Send/Recv becomes one kernel; other p2p-based
      // collectives run alone.
      size_t j = i + 1;
      if (isP2pKind(h.kind))
        while (j < ops.size() && isP2pKind(ops[j].kind)) j++;
      cudaStream_t s = ops[i].stream;
      bool anySync = false;
      // Order every stream of the run before the kernel and after it (the
      // events are destroyed on every exit; a destroyed event that a stream
      // still waits on completes as recorded).
      struct Events {
        std::vector<cudaEvent_t> v;
        ~Events() {
          for (cudaEvent_t e : v) cudaEventDestroy(e);
        }
      } evs;
      std::vector<cudaStream_t> others;  // the run's streams other than s (each op is moved onto s below)
      for (size_t k = i; k < j; k++) {
        if (ops[k].stream != s && std::find(others.begin(), others.end(), ops[k].stream) == others.end()) {
          others.push_back(ops[k].stream);
          cudaEvent_t ev = nullptr;
          VTRY(cudaToVccl(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event"));
          evs.v.push_back(ev);
          VTRY(cudaToVccl(cudaEventRecord(ev, ops[k].stream), "event record"));
          VTRY(cudaToVccl(cudaStreamWaitEvent(s, ev, 0), "stream wait"));
        }
      }
      OrderedLaunch ord(comm->dev.get(), s);
      PlanBuilder pb;
      for (size_t k = i; k < j; k++) {
        ops[k].stream = s;
        VTRY(prepareBuffers(ops[k], st));
        VTRY(addP2pWork(ops[k], pb));
        anySync |= ops[k].sync;
      }
      VTRY(pb.finalize());
      VTRY(cudaToVccl(launchP2p(launchCtx(comm, s), pb.plan), "point-to-point launch"));
      VTRY(st.finish(s));
      for (size_t k = i; k < j; k++) comm->noteCall(opName(ops[k].kind), "point-to-point kernel", callBytes(ops[k]));
      if (!others.empty()) {
        cudaEvent_t done = nullptr;
        VTRY(cudaToVccl(cudaEventCreateWithFlags(&done, cudaEventDisableTiming), "event"));
        evs.v.push_back(done);
        VTRY(cudaToVccl(cudaEventRecord(done, s), "event record"));
        for (cudaStream_t o : others) VTRY(cudaToVccl(cudaStreamWaitEvent(o, done, 0), "stream wait"));
      }
      if (anySync) waits->push_back({comm, s});
      i = j;
      continue;
    }
    OrderedLaunch ord(comm->dev.get(), h.stream);
    VTRY(prepareBuffers(h, st));
    if (comm->dev->regCacheOn && comm->nranks > 1) VTRY(cacheWindowsFor(h, st.ranges.empty()));
    tAlgo = nullptr;
    VTRY(launchColl(h));
    VTRY(st.finish(h.stream));
    comm->noteCall(opName(h.kind), tAlgo ? tAlgo : comm->nranks == 1 ? "local copy" : "two-shot to root",
                   callBytes(h));
    if (h.sync) waits->push_back({comm, h.stream});
    i++;
  }
  return vcclSuccess;
}

vcclResult_t waitAll(const std::vector<PendingSync>& waits) {
  vcclResult_t res = vcclSuccess;
  for (const PendingSync& w : waits) {
    cudaSetDevice(w.comm->dev->device);
    cudaError_t e = cudaStreamSynchronize(w.stream);
    vcclResult_t r = w.comm->pollDeviceStatus();
    if (r == vcclSuccess && e != cudaSuccess) {
      VERR("stream synchronize failed: %s", cudaGetErrorString(e));
      r = vcclUnhandledError;
    }
    if (r != vcclSuccess) {
      w.comm->noteError(r);
      if (res == vcclSuccess) res = r;
    }
  }
  return res;
}

vcclResult_t submit(HostOp&& h) {
  if (tDepth > 0) {
    tQueue.push_back(std::move(h));
    return vcclSuccess;
  }
  vcclComm_t comm = h.comm;
  std::vector<HostOp> ops;
  ops.push_back(std::move(h));
  std::vector<PendingSync> waits;
  vcclResult_t r = launchOps(comm, ops, &waits);
  if (r != vcclSuccess) {
    comm->noteError(r);
    // Launched work must still finish before we report.
    waitAll(waits);
    return r;
  }
  r = waitAll(waits);
  return r;
}

// Common construction of a HostOp for a call.
HostOp makeOp(Kind k, vcclComm_t comm, const void* send, void* recv, size_t count, vcclDataType_t dt,
              vcclStream_t stream, bool async) {
  HostOp h;
  h.kind = k;
  h.comm = comm;
  h.send = static_cast<const char*>(send);
  h.recv = static_cast<char*>(recv);
  h.count = count;
  h.dt = dt;
  if (async) {
    h.stream = reinterpret_cast<cudaStream_t>(stream);
    h.sync = false;
    h.staged = false;
  } else {
    h.stream = cudaStreamLegacy;
    h.sync = comm->blocking;
    h.staged = true;
  }
  return h;
}

vcclResult_t baseChecks(vcclComm_t comm, vcclDataType_t dt) {
  VTRY(usable(comm));
  if (vcclTypeSize(dt) == 0) return vcclInvalidArgument;
  return vcclSuccess;
}

vcclResult_t doAllReduce(const void* send, void* recv, size_t count, vcclDataType_t dt, vcclRedOp_t op,
                         vcclComm_t comm, vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (send == nullptr || recv == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::AllReduce, comm, send, recv, count, dt, stream, async);
  VTRY(resolveOp(comm, dt, op, &h));
  return submit(std::move(h));
}

vcclResult_t doReduce(const void* send, void* recv, size_t count, vcclDataType_t dt, vcclRedOp_t op, int root,
                      vcclComm_t comm, vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (send == nullptr || root < 0 || root >= comm->nranks) return vcclInvalidArgument;
  if (comm->rank == root && recv == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::Reduce, comm, send, recv, count, dt, stream, async);
  h.root = root;
  VTRY(resolveOp(comm, dt, op, &h));
  return submit(std::move(h));
}

vcclResult_t doReduceScatter(const void* send, void* recv, size_t rc, vcclDataType_t dt, vcclRedOp_t op,
                             vcclComm_t comm, vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (send == nullptr || recv == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::ReduceScatter, comm, send, recv, rc, dt, stream, async);
  VTRY(resolveOp(comm, dt, op, &h));
  if (comm->nranks == 1 || rc == 0) {
    // One rank: the single chunk is this rank's own block.
  } else {
    // Reduce-scatter reads chunk `rank` of send for the local contribution;
    // nothing else to adjust here.
  }
  return submit(std::move(h));
}

vcclResult_t doAllGather(const void* send, void* recv, size_t sc, vcclDataType_t dt, vcclComm_t comm,
                         vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (send == nullptr || recv == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::AllGather, comm, send, recv, sc, dt, stream, async);
  if (comm->nranks == 1) return submit(std::move(h));
  return submit(std::move(h));
}

vcclResult_t doBroadcast(const void* send, void* recv, size_t count, vcclDataType_t dt, int root,
                         vcclComm_t comm, vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (recv == nullptr || root < 0 || root >= comm->nranks) return vcclInvalidArgument;
  if (comm->rank == root && send == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::Broadcast, comm, comm->rank == root ? send : recv, recv, count, dt, stream, async);
  h.root = root;
  return submit(std::move(h));
}

vcclResult_t doGather(const void* send, void* recv, size_t sc, vcclDataType_t dt, int root, vcclComm_t comm,
                      vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (send == nullptr || root < 0 || root >= comm->nranks) return vcclInvalidArgument;
  if (comm->rank == root && recv == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::Gather, comm, send, recv, sc, dt, stream, async);
  h.root = root;
  return submit(std::move(h));
}

vcclResult_t doScatter(const void* send, void* recv, size_t rc, vcclDataType_t dt, int root, vcclComm_t comm,
                       vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (recv == nullptr || root < 0 || root >= comm->nranks) return vcclInvalidArgument;
  if (comm->rank == root && send == nullptr) return vcclInvalidArgument;
  HostOp h = makeOp(Kind::Scatter, comm, send, recv, rc, dt, stream, async);
  h.root = root;
  return submit(std::move(h));
}

vcclResult_t doAllToAllv(const void* send, const size_t* sc, const size_t* sd, void* recv, const size_t* rc,
                         const size_t* rd, vcclDataType_t dt, vcclComm_t comm, vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (send == nullptr || recv == nullptr || sc == nullptr || sd == nullptr || rc == nullptr || rd == nullptr)
    return vcclInvalidArgument;
  HostOp h = makeOp(Kind::AllToAllv, comm, send, recv, 0, dt, stream, async);
  const int n = comm->nranks;
  h.sc.assign(sc, sc + n);
  h.sd.assign(sd, sd + n);
  h.rc.assign(rc, rc + n);
  h.rd.assign(rd, rd + n);
  return submit(std::move(h));
}

vcclResult_t doP2p(bool isSend, const void* buf, size_t count, vcclDataType_t dt, int peer, vcclComm_t comm,
                   vcclStream_t stream, bool async) {
  VTRY(baseChecks(comm, dt));
  if (buf == nullptr || peer < 0 || peer >= comm->nranks || peer == comm->rank) return vcclInvalidArgument;
  HostOp h = makeOp(isSend ? Kind::Send : Kind::Recv, comm, isSend ? buf : nullptr,
                    isSend ? nullptr : const_cast<void*>(buf), count, dt, stream, async);
  h.peer = peer;
  return submit(std::move(h));
}

}  // namespace
}  // namespace vccl

using namespace vccl;

extern "C" {

vcclResult_t vcclGroupStart(void) {
  tDepth++;
  return vcclSuccess;
}

vcclResult_t vcclGroupEnd(void) {
  if (tDepth == 0) return vcclInvalidUsage;
  if (--tDepth > 0) return vcclSuccess;
  std::vector<HostOp> all;
  all.swap(tQueue);
  if (all.empty()) return vcclSuccess;
  std::vector<vcclComm_t> order;
  std::map<vcclComm_t, std::vector<HostOp>> byComm;
  for (HostOp& h : all) {
    if (byComm.find(h.comm) == byComm.end()) order.push_back(h.comm);
    byComm[h.comm].push_back(std::move(h));
  }
  // Launch everything first (communicators of one process wait on each
  // other), then wait.
  std::vector<PendingSync> waits;
  vcclResult_t first = vcclSuccess;
  // Communicators without a device run their calls on the host, blocking
  // until the peers take part: when one group holds several of them (ranks
  // of one process, vcclCommInitAll), each runs on its own thread so they
  // can meet.
  std::vector<vcclComm_t> hostComms;
  for (vcclComm_t c : order)
    if (!c->dev && c->nranks > 1) hostComms.push_back(c);
  std::vector<vcclResult_t> hostRes(hostComms.size(), vcclSuccess);
  std::vector<std::thread> hostThreads;
  if (hostComms.size() > 1)
    for (size_t i = 0; i < hostComms.size(); i++)
      hostThreads.emplace_back([&, i] { hostRes[i] = launchOps(hostComms[i], byComm[hostComms[i]], nullptr); });
  for (vcclComm_t c : order) {
    if (hostComms.size() > 1 && !c->dev && c->nranks > 1) continue;
    vcclResult_t r = launchOps(c, byComm[c], &waits);
    if (r != vcclSuccess) {
      c->noteError(r);
      if (first == vcclSuccess) first = r;
    }
  }
  for (size_t i = 0; i < hostThreads.size(); i++) {
    hostThreads[i].join();
    if (hostRes[i] != vcclSuccess) {
      hostComms[i]->noteError(hostRes[i]);
      if (first == vcclSuccess) first = hostRes[i];
    }
  }
  vcclResult_t w = waitAll(waits);
  return first != vcclSuccess ? first : w;
}

vcclResult_t vcclAllReduce(const void* s, void* r, size_t n, vcclDataType_t dt, vcclRedOp_t op, vcclComm_t c) {
  return doAllReduce(s, r, n, dt, op, c, nullptr, false);
}
vcclResult_t vcclAllReduceAsync(const void* s, void* r, size_t n, vcclDataType_t dt, vcclRedOp_t op, vcclComm_t c,
                                vcclStream_t st) {
  return doAllReduce(s, r, n, dt, op, c, st, true);
}
vcclResult_t vcclReduce(const void* s, void* r, size_t n, vcclDataType_t dt, vcclRedOp_t op, int root,
                        vcclComm_t c) {
  return doReduce(s, r, n, dt, op, root, c, nullptr, false);
}
vcclResult_t vcclReduceAsync(const void* s, void* r, size_t n, vcclDataType_t dt, vcclRedOp_t op, int root,
                             vcclComm_t c, vcclStream_t st) {
  return doReduce(s, r, n, dt, op, root, c, st, true);
}
vcclResult_t vcclReduceScatter(const void* s, void* r, size_t n, vcclDataType_t dt, vcclRedOp_t op,
                               vcclComm_t c) {
  return doReduceScatter(s, r, n, dt, op, c, nullptr, false);
}
vcclResult_t vcclReduceScatterAsync(const void* s, void* r, size_t n, vcclDataType_t dt, vcclRedOp_t op,
                                    vcclComm_t c, vcclStream_t st) {
  return doReduceScatter(s, r, n, dt, op, c, st, true);
}
vcclResult_t vcclAllGather(const void* s, void* r, size_t n, vcclDataType_t dt, vcclComm_t c) {
  return doAllGather(s, r, n, dt, c, nullptr, false);
}
vcclResult_t vcclAllGatherAsync(const void* s, void* r, size_t n, vcclDataType_t dt, vcclComm_t c,
                                vcclStream_t st) {
  return doAllGather(s, r, n, dt, c, st, true);
}
vcclResult_t vcclBroadcast(const void* s, void* r, size_t n, vcclDataType_t dt, int root, vcclComm_t c) {
  return doBroadcast(s, r, n, dt, root, c, nullptr, false);
}
vcclResult_t vcclBroadcastAsync(const void* s, void* r, size_t n, vcclDataType_t dt, int root, vcclComm_t c,
                                vcclStream_t st) {
  return doBroadcast(s, r, n, dt, root, c, st, true);
}
vcclResult_t vcclBcast(void* b, size_t n, vcclDataType_t dt, int root, vcclComm_t c) {
  return doBroadcast(b, b, n, dt, root, c, nullptr, false);
}
vcclResult_t vcclGather(const void* s, void* r, size_t n, vcclDataType_t dt, int root, vcclComm_t c) {
  return doGather(s, r, n, dt, root, c, nullptr, false);
}
vcclResult_t vcclGatherAsync(const void* s, void* r, size_t n, vcclDataType_t dt, int root, vcclComm_t c,
                             vcclStream_t st) {
  return doGather(s, r, n, dt, root, c, st, true);
}
vcclResult_t vcclScatter(const void* s, void* r, size_t n, vcclDataType_t dt, int root, vcclComm_t c) {
  return doScatter(s, r, n, dt, root, c, nullptr, false);
}
vcclResult_t vcclScatterAsync(const void* s, void* r, size_t n, vcclDataType_t dt, int root, vcclComm_t c,
                              vcclStream_t st) {
  return doScatter(s, r, n, dt, root, c, st, true);
}
vcclResult_t vcclAllToAll(const void* s, void* r, size_t n, vcclDataType_t dt, vcclComm_t c) {
  if (c == nullptr) return vcclInvalidArgument;
  std::vector<size_t> cnt(c->nranks, n), dis(c->nranks);
  for (int i = 0; i < c->nranks; i++) dis[i] = i * n;
  return doAllToAllv(s, cnt.data(), dis.data(), r, cnt.data(), dis.data(), dt, c, nullptr, false);
}
vcclResult_t vcclAllToAllAsync(const void* s, void* r, size_t n, vcclDataType_t dt, vcclComm_t c,
                               vcclStream_t st) {
  if (c == nullptr) return vcclInvalidArgument;
  std::vector<size_t> cnt(c->nranks, n), dis(c->nranks);
  for (int i = 0; i < c->nranks; i++) dis[i] = i * n;
  return doAllToAllv(s, cnt.data(), dis.data(), r, cnt.data(), dis.data(), dt, c, st, true);
}
vcclResult_t vcclAllToAllv(const void* s, const size_t sc[], const size_t sd[], void* r, const size_t rc[],
                           const size_t rd[], vcclDataType_t dt, vcclComm_t c) {
  return doAllToAllv(s, sc, sd, r, rc, rd, dt, c, nullptr, false);
}
vcclResult_t vcclAllToAllvAsync(const void* s, const size_t sc[], const size_t sd[], void* r, const size_t rc[],
                                const size_t rd[], vcclDataType_t dt, vcclComm_t c, vcclStream_t st) {
  return doAllToAllv(s, sc, sd, r, rc, rd, dt, c, st, true);
}
vcclResult_t vcclSend(const void* b, size_t n, vcclDataType_t dt, int peer, vcclComm_t c) {
  return doP2p(true, b, n, dt, peer, c, nullptr, false);
}
vcclResult_t vcclSendAsync(const void* b, size_t n, vcclDataType_t dt, int peer, vcclComm_t c, vcclStream_t st) {
  return doP2p(true, b, n, dt, peer, c, st, true);
}
vcclResult_t vcclRecv(void* b, size_t n, vcclDataType_t dt, int peer, vcclComm_t c) {
  return doP2p(false, b, n, dt, peer, c, nullptr, false);
}
vcclResult_t vcclRecvAsync(void* b, size_t n, vcclDataType_t dt, int peer, vcclComm_t c, vcclStream_t st) {
  return doP2p(false, b, n, dt, peer, c, st, true);
}

}  // extern "C"
