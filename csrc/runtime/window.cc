// SPDX-License-Identifier: Apache-2.0
// Window registration: map a user buffer into every rank of the communicator.
//
// The reference's vcclCommRegister pins a buffer for its own transport and
// is a local call (reference: src/core/comm.cc:180-244); vcclCommRegister
// keeps that meaning here.  vcclCommWindowRegister is the collective
// counterpart that lets kernels touch the buffer from every GPU.  For a
// buffer inside a vcclMemAlloc allocation each rank exports the VMM handle,
// the handles travel over the bootstrap's Unix sockets (SCM_RIGHTS, like
// the workspaces), every rank maps every peer's allocation, and when the
// node supports NVLS the windows are also bound to one multicast object.
// A buffer from plain cudaMalloc (a PyTorch tensor, say) goes through CUDA
// IPC instead: its allocation's IPC handle is all-gathered and every rank
// opens the peers' handles (ranks of the same process, from
// vcclCommInitAll, use each other's pointers directly with peer access
// enabled); such windows have no multicast binding.
// Collectives whose buffers lie in windows then run the zero-copy kernels of
// csrc/kernels/window.cuh.
//
// The registration cache (VCCL_REG_CACHE=1) registers such windows on demand
// for plain device buffers of large collectives and keeps them: the
// NVLink form of the reference's per-call registration with an LRU cache
// (reference: src/core/comm.h:74-139).  Its decisions are made in
// runtime/regcache.cc from one allgather per call.
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <vector>

#include "common/env.h"
#include "common/log.h"
#include "common/net.h"
#include "runtime/comm.h"
#include "runtime/cudrv.h"

namespace vccl {

namespace {

size_t roundUpTo(size_t x, size_t a) { return (x + a - 1) / a * a; }

enum WinKind : uint32_t { kWinNone = 0, kWinVmm = 1, kWinIpc = 2 };

struct WinInfo {
  uint64_t size;        // window bytes
  uint64_t offset;      // window offset inside the rank's allocation
  uint64_t allocBytes;  // the rank's allocation
  uint32_t kind;        // WinKind
  int32_t pid;
  int32_t device;       // CUDA device of the rank
  int32_t pad;
  uint64_t rawBase;     // kWinIpc: the allocation's address in its own process
  cudaIpcMemHandle_t ipc;  // kWinIpc: handle of the allocation
};

// Bind every rank's window to one multicast object (rank 0 creates it).
// Every rank takes the same steps; false on all ranks if any step failed
// anywhere, with nothing left bound.
bool windowMulticast(Bootstrap* bs, DeviceState* ds, Window* w, const std::vector<WinInfo>& info) {
  const DriverApi* d = driverApi();
  const int n = bs->nranks(), me = bs->rank();
  CUmulticastObjectProp mp;
  memset(&mp, 0, sizeof(mp));
  mp.numDevices = static_cast<unsigned int>(n);
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  mp.size = w->bytes;
  size_t gran = 0;
  bool ok = d->mcGranularity(&gran, &mp, CU_MULTICAST_GRANULARITY_MINIMUM) == CUDA_SUCCESS && gran > 0;
  // The bound range must start at a multiple of the granularity inside the
  // allocation and fit in it once rounded up.
  const size_t mcBytes = ok ? roundUpTo(w->bytes, gran) : 0;
  ok = ok && info[me].offset % gran == 0 && info[me].offset + mcBytes <= info[me].allocBytes;
  if (!everyone(bs, ok)) return false;
  mp.size = mcBytes;
  w->mcBytes = mcBytes;
  int fd = -1;
  if (me == 0)
    ok = d->mcCreate(&w->mcHandle, &mp) == CUDA_SUCCESS &&
         d->memExport(&fd, w->mcHandle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) == CUDA_SUCCESS;
  if (!everyone(bs, ok)) {
    closeFd(fd);
    windowReleaseMulticast(ds, w);
    return false;
  }
  std::vector<int> fds;
  if (me == 0) fds.push_back(fd);
  if (bs->broadcastFds(0, &fds, 1) != vcclSuccess) {
    if (me == 0) closeFd(fd);
    windowReleaseMulticast(ds, w);
    return false;
  }
  if (me == 0) {
    closeFd(fd);
  } else {
    ok = fds.size() == 1 && d->memImport(&w->mcHandle, reinterpret_cast<void*>(static_cast<uintptr_t>(fds[0])),
                                         CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
    for (int f : fds) closeFd(f);
  }
  ok = ok && d->mcAddDevice(w->mcHandle, ds->cuDevice) == CUDA_SUCCESS;
  // Every device must be added before any memory is bound.
  if (!everyone(bs, ok)) {
    windowReleaseMulticast(ds, w);
    return false;
  }
  const CUresult br = d->mcBindMem(w->mcHandle, 0, w->localHandle, w->localOffset, mcBytes, 0);
  ok = br == CUDA_SUCCESS;
  if (!ok) VWARN("window: cuMulticastBindMem failed: %s", cuErrorText(br));
  w->mcBound = ok;
  if (!everyone(bs, ok)) {
    windowReleaseMulticast(ds, w);
    return false;
  }
  ok = mapForDevice(d, w->mcHandle, mcBytes, gran, ds->device, &w->mcVa) == vcclSuccess;
  if (!everyone(bs, ok)) {
    windowReleaseMulticast(ds, w);
    return false;
  }
  w->mc = reinterpret_cast<char*>(w->mcVa);
  return true;
}

}  // namespace

void windowReleaseMulticast(DeviceState* ds, Window* w) {
  const DriverApi* d = driverApi();
  if (d == nullptr) return;
  if (w->mcVa) {
    d->memUnmap(w->mcVa, w->mcBytes);
    d->memAddressFree(w->mcVa, w->mcBytes);
    w->mcVa = 0;
  }
  if (w->mcBound) {
    d->mcUnbind(w->mcHandle, ds->cuDevice, 0, w->mcBytes);
    w->mcBound = false;
  }
  if (w->mcHandle) {
    d->memRelease(w->mcHandle);
    w->mcHandle = 0;
  }
  w->mc = nullptr;
}

void windowRelease(DeviceState* ds, int me, Window* w) {
  const DriverApi* d = driverApi();
  if (d == nullptr) return;
  windowReleaseMulticast(ds, w);
  for (size_t p = 0; p < w->ipcBase.size(); p++) {
    if (static_cast<int>(p) != me && w->ipcBase[p] != nullptr) cudaIpcCloseMemHandle(w->ipcBase[p]);
    w->ipcBase[p] = nullptr;
  }
  for (size_t p = 0; p < w->peerVa.size(); p++) {
    if (static_cast<int>(p) == me) continue;
    if (w->peerVa[p]) {
      d->memUnmap(w->peerVa[p], w->peerVaBytes[p]);
      d->memAddressFree(w->peerVa[p], w->peerVaBytes[p]);
      w->peerVa[p] = 0;
    }
    if (w->peerHandle[p]) {
      d->memRelease(w->peerHandle[p]);
      w->peerHandle[p] = 0;
    }
  }
}

vcclResult_t windowRegister(vcclComm_t comm, void* buff, size_t size, int flags, bool cached, Window** win) {
  if (comm == nullptr || buff == nullptr || size == 0 || win == nullptr) return vcclInvalidArgument;
  if (comm->aborted.load()) return vcclInvalidUsage;
  if (!comm->dev || driverApi() == nullptr) {
    VERR("vcclCommWindowRegister: the communicator has no device data plane");
    return vcclInvalidUsage;
  }
  Bootstrap* bs = comm->bootstrap.get();
  DeviceState* ds = comm->dev.get();
  const DriverApi* d = driverApi();
  const int n = comm->nranks, me = comm->rank;
  cudaSetDevice(ds->device);

  void* allocBase = nullptr;
  size_t allocBytes = 0;
  CUmemGenericAllocationHandle h = 0;
  std::vector<WinInfo> info(n);
  WinInfo& mine = info[me];
  memset(&mine, 0, sizeof(mine));
  mine.size = size;
  mine.pid = static_cast<int32_t>(getpid());
  mine.device = ds->device;
  if (findDeviceAllocation(buff, size, &allocBase, &allocBytes, &h)) {
    mine.kind = kWinVmm;
  } else {
    // Plain device memory: the allocation around the buffer, by IPC handle.
    CUdeviceptr base = 0;
    size_t bytes = 0;
    if (d->memGetAddressRange(&base, &bytes, reinterpret_cast<CUdeviceptr>(buff)) == CUDA_SUCCESS &&
        reinterpret_cast<CUdeviceptr>(buff) + size <= base + bytes &&
        cudaIpcGetMemHandle(&mine.ipc, reinterpret_cast<void*>(base)) == cudaSuccess) {
      mine.kind = kWinIpc;
      mine.rawBase = static_cast<uint64_t>(base);
      allocBase = reinterpret_cast<void*>(base);
      allocBytes = bytes;
    }
    cudaGetLastError();
  }
  mine.offset = mine.kind ? static_cast<uint64_t>(static_cast<char*>(buff) - static_cast<char*>(allocBase)) : 0;
  mine.allocBytes = allocBytes;
  vcclResult_t res = bs->allGather(info.data(), sizeof(WinInfo));
  if (res != vcclSuccess) return res;
  for (int p = 0; p < n; p++) {
    if (info[p].kind == kWinNone) {
      VERR("vcclCommWindowRegister: rank %d's buffer is neither vcclMemAlloc nor cudaMalloc device memory", p);
      return vcclInvalidArgument;
    }
    if (info[p].kind != info[0].kind) {
      VERR("vcclCommWindowRegister: every rank must pass the same kind of memory (vcclMemAlloc or cudaMalloc)");
      return vcclInvalidArgument;
    }
    if (info[p].size != size) {
      VERR("vcclCommWindowRegister: window sizes differ (%zu on rank %d, %zu here)",
           static_cast<size_t>(info[p].size), p, size);
      return vcclInvalidArgument;
    }
  }

  auto w = std::make_unique<Window>();
  w->base = static_cast<char*>(buff);
  w->bytes = size;
  w->localHandle = h;
  w->localOffset = info[me].offset;
  w->peer.assign(n, nullptr);
  w->peerVa.assign(n, 0);
  w->peerVaBytes.assign(n, 0);
  w->peerHandle.assign(n, 0);
  w->ipcBase.assign(n, nullptr);
  w->peer[me] = w->base;
  w->cached = cached;

  if (mine.kind == kWinIpc) {
    bool ok = true;
    for (int p = 0; p < n && ok; p++) {
      if (p == me) continue;
      if (info[p].pid == mine.pid) {
        // Same process (vcclCommInitAll): the peer's pointer is valid here
        // once this device may access the peer's.
        const cudaError_t pe = cudaDeviceEnablePeerAccess(info[p].device, 0);
        ok = pe == cudaSuccess || pe == cudaErrorPeerAccessAlreadyEnabled;
        if (ok) w->peer[p] = reinterpret_cast<char*>(info[p].rawBase) + info[p].offset;
        continue;
      }
      ok = cudaIpcOpenMemHandle(&w->ipcBase[p], info[p].ipc, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
      if (ok) w->peer[p] = static_cast<char*>(w->ipcBase[p]) + info[p].offset;
    }
    cudaGetLastError();
    if (!everyone(bs, ok)) {
      windowRelease(ds, me, w.get());
      VERR("vcclCommWindowRegister: opening a peer's IPC handle failed on some rank");
      return vcclSystemError;
    }
    res = bs->barrier();
    if (res != vcclSuccess) {
      windowRelease(ds, me, w.get());
      return res;
    }
    VINFO("window registered: %zu bytes of cudaMalloc memory, point-to-point%s", size,
          cached ? " (registration cache)" : "");
    std::lock_guard<std::mutex> g(comm->regMu);
    comm->windows.push_back(w.get());
    *win = w.release();
    return vcclSuccess;
  }

  int fd = -1;
  bool ok = d->memExport(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) == CUDA_SUCCESS;
  if (!everyone(bs, ok)) {
    closeFd(fd);
    VERR("vcclCommWindowRegister: exporting the allocation failed on some rank");
    return vcclSystemError;
  }
  std::vector<std::vector<int>> fds;
  res = bs->exchangeFds({fd}, &fds);
  closeFd(fd);
  if (res != vcclSuccess) return res;
  for (int p = 0; p < n; p++) {
    if (p != me && ok) {
      ok = fds[p].size() == 1 &&
           d->memImport(&w->peerHandle[p], reinterpret_cast<void*>(static_cast<uintptr_t>(fds[p][0])),
                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
      if (ok) {
        w->peerVaBytes[p] = info[p].allocBytes;
        ok = mapForDevice(d, w->peerHandle[p], info[p].allocBytes, ds->gran, ds->device, &w->peerVa[p]) ==
             vcclSuccess;
      }
      if (ok) w->peer[p] = reinterpret_cast<char*>(w->peerVa[p]) + info[p].offset;
    }
    for (int f : fds[p]) closeFd(f);
  }
  if (!everyone(bs, ok)) {
    windowRelease(ds, me, w.get());
    VERR("vcclCommWindowRegister: mapping a peer's window failed on some rank");
    return vcclSystemError;
  }
  const bool wantMc = ds->nvls && (flags & VCCL_WIN_NO_MULTICAST) == 0 && envLong("VCCL_WINDOW_NVLS", 1) != 0;
  // The flags and VCCL_WINDOW_NVLS are per rank; the ranks agree first, so
  // that all of them take (or skip) the multicast steps together.
  if (everyone(bs, wantMc) && !windowMulticast(bs, ds, w.get(), info))
    VINFO("window of %zu bytes: no multicast binding, point-to-point only", size);
  res = bs->barrier();
  if (res != vcclSuccess) {
    windowRelease(ds, me, w.get());
    return res;
  }
  VINFO("window registered: %zu bytes, %s", size, w->mc ? "multicast bound" : "point-to-point");
  std::lock_guard<std::mutex> g(comm->regMu);
  comm->windows.push_back(w.get());
  *win = w.release();
  return vcclSuccess;
}

namespace {

// Drop one window everywhere: every rank's kernels are done with it before
// any rank unmaps (collective).
vcclResult_t windowDrop(vcclComm_t comm, Window* w) {
  {
    std::lock_guard<std::mutex> g(comm->regMu);
    auto it = std::find(comm->windows.begin(), comm->windows.end(), w);
    if (it == comm->windows.end()) return vcclInvalidArgument;
    comm->windows.erase(it);
  }
  vcclResult_t res = vcclSuccess;
  if (comm->dev) {
    cudaSetDevice(comm->dev->device);
    cudaDeviceSynchronize();  // this rank's kernels are done with the window
    // ... and so are the peers' once everyone got here; an aborted
    // communicator skips the meeting (its peers may be gone).
    if (!comm->aborted.load()) res = comm->bootstrap->barrier();
    windowRelease(comm->dev.get(), comm->rank, w);
  }
  delete w;
  return res;
}

}  // namespace

// The registration cache's device side.  Everything that decides is in
// RegCacheBook (runtime/regcache.cc); this part gathers each rank's facts
// (allocation ids from the driver, capture state, application windows),
// runs the one allgather per call and carries out the plan with the window
// steps above.
vcclResult_t regCacheWindows(vcclComm_t comm, cudaStream_t s, const void* const* ptrs, const size_t* bytes,
                             int nbuf, bool eligible, const Window** out) {
  for (int i = 0; i < nbuf; i++) out[i] = nullptr;
  if (nbuf < 1 || nbuf > kRegMaxBuffers) return vcclInternalError;
  const DriverApi* d = driverApi();
  std::lock_guard<std::mutex> cacheLock(comm->regCacheMu);
  RegKey keys[kRegMaxBuffers];
  bool ok = eligible && d != nullptr && d->pointerGetAttribute != nullptr && !comm->aborted.load();
  if (ok) {
    // Registering blocks the host and dropping synchronizes the device: not
    // while the stream is being captured (the call then stays staged, on
    // every rank, through the plan).
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) ok = false;
    cudaGetLastError();
  }
  for (int i = 0; i < nbuf && ok; i++) {
    keys[i].ptr = reinterpret_cast<uintptr_t>(ptrs[i]);
    keys[i].bytes = bytes[i];
    keys[i].userWindow = comm->findWindow(ptrs[i], bytes[i]) != nullptr;
    if (keys[i].userWindow) continue;
    // Only memory that CUDA IPC can export (cudaMalloc; not the stream-ordered
    // pool, not VMM ranges, which vcclMemAlloc + vcclCommWindowRegister serve).
    // The driver writes a boolean for the IPC attribute; a zeroed 8-byte
    // slot reads nonzero exactly when it wrote true, whatever its width.
    unsigned long long id = 0, ipcOk = 0;
    const CUdeviceptr p = reinterpret_cast<CUdeviceptr>(ptrs[i]);
    ok = d->pointerGetAttribute(&id, CU_POINTER_ATTRIBUTE_BUFFER_ID, p) == CUDA_SUCCESS &&
         d->pointerGetAttribute(&ipcOk, CU_POINTER_ATTRIBUTE_IS_LEGACY_CUDA_IPC_CAPABLE, p) == CUDA_SUCCESS &&
         ipcOk != 0 && id != 0;
    keys[i].allocId = id;
  }
  if (ok && nbuf == 2 && keys[0].ptr < keys[1].ptr + keys[1].bytes && keys[1].ptr < keys[0].ptr + keys[0].bytes)
    ok = false;  // overlapping send and receive ranges (in-place forms pass one buffer)
  cudaGetLastError();

  const int n = comm->nranks, me = comm->rank;
  std::vector<RegQuery> all(n);
  all[me] = comm->regCache.query(keys, nbuf, ok);
  VTRY(comm->bootstrap->allGather(all.data(), sizeof(RegQuery)));
  const RegPlan plan = comm->regCache.plan(all);
  comm->regCache.countCall(plan);
  if (!plan.take) return vcclSuccess;
  for (int32_t id : plan.evict) VTRY(windowDrop(comm, static_cast<Window*>(comm->regCache.drop(id))));
  for (int i = 0; i < nbuf; i++) {
    if (plan.use[i] >= 0) {
      comm->regCache.touch(plan.use[i]);
      out[i] = static_cast<const Window*>(comm->regCache.handleOf(plan.use[i]));
      continue;
    }
    if (!plan.reg[i]) continue;
    Window* w = nullptr;
    const vcclResult_t r = windowRegister(comm, const_cast<void*>(ptrs[i]), bytes[i], VCCL_WIN_NO_MULTICAST, true, &w);
    if (r != vcclSuccess) {
      // Registration fails on every rank alike (its steps agree through the
      // bootstrap), so every rank turns the cache off here and the call, with
      // every later one, stays on the staged kernels.
      VWARN("registration cache: registering a %zu-byte buffer failed (%s); cache off for this communicator",
            bytes[i], vcclGetErrorString(r));
      comm->dev->regCacheOn = false;
      for (int j = 0; j < nbuf; j++) out[j] = nullptr;
      return vcclSuccess;
    }
    comm->regCache.add(keys[i], w);
    out[i] = w;
  }
  return vcclSuccess;
}

vcclResult_t regCacheFlush(vcclComm_t comm) {
  std::lock_guard<std::mutex> cacheLock(comm->regCacheMu);
  vcclResult_t res = vcclSuccess;
  for (int32_t id : comm->regCache.ids()) {
    const vcclResult_t r = windowDrop(comm, static_cast<Window*>(comm->regCache.drop(id)));
    if (res == vcclSuccess) res = r;
  }
  return res;
}

}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclCommWindowRegister(vcclComm_t comm, void* buff, size_t size, vcclWindow_t* win,
                                               int flags) {
  if (win == nullptr) return vcclInvalidArgument;
  Window* w = nullptr;
  const vcclResult_t r = windowRegister(comm, buff, size, flags, false, &w);
  if (r == vcclSuccess) *win = w;
  return r;
}

extern "C" vcclResult_t vcclCommWindowDeregister(vcclComm_t comm, vcclWindow_t win) {
  if (comm == nullptr || win == nullptr) return vcclInvalidArgument;
  Window* w = static_cast<Window*>(win);
  {
    // Cached windows belong to the registration cache, not to the caller.
    std::lock_guard<std::mutex> g(comm->regMu);
    if (std::find(comm->windows.begin(), comm->windows.end(), w) == comm->windows.end() || w->cached)
      return vcclInvalidArgument;
  }
  return windowDrop(comm, w);
}

extern "C" vcclResult_t vcclCommRegCacheFlush(vcclComm_t comm) {
  if (comm == nullptr) return vcclInvalidArgument;
  if (!comm->dev) return vcclSuccess;
  return regCacheFlush(comm);
}

extern "C" vcclResult_t vcclCommRegCacheStats(vcclComm_t comm, unsigned long long* out) {
  if (comm == nullptr || out == nullptr) return vcclInvalidArgument;
  std::lock_guard<std::mutex> cacheLock(comm->regCacheMu);
  const RegStats& st = comm->regCache.stats();
  out[0] = comm->regCache.entries().size();
  out[1] = st.calls;
  out[2] = st.hits;
  out[3] = st.misses;
  out[4] = st.evictions;
  out[5] = static_cast<unsigned long long>(comm->regCache.capacity());
  return vcclSuccess;
}
