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

}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclCommWindowRegister(vcclComm_t comm, void* buff, size_t size, vcclWindow_t* win,
                                               int flags) {
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
    VINFO("window registered: %zu bytes of cudaMalloc memory, point-to-point", size);
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

extern "C" vcclResult_t vcclCommWindowDeregister(vcclComm_t comm, vcclWindow_t win) {
  if (comm == nullptr || win == nullptr) return vcclInvalidArgument;
  Window* w = static_cast<Window*>(win);
  {
    std::lock_guard<std::mutex> g(comm->regMu);
    auto it = std::find(comm->windows.begin(), comm->windows.end(), w);
    if (it == comm->windows.end()) return vcclInvalidArgument;
    comm->windows.erase(it);
  }
  vcclResult_t res = vcclSuccess;
  if (comm->dev) {
    cudaSetDevice(comm->dev->device);
    cudaDeviceSynchronize();  // this rank's kernels are done with every window
    // ... and so are the peers' once everyone got here; an aborted
    // communicator skips the meeting (its peers may be gone).
    if (!comm->aborted.load()) res = comm->bootstrap->barrier();
    windowRelease(comm->dev.get(), comm->rank, w);
  }
  delete w;
  return res;
}
