// SPDX-License-Identifier: Apache-2.0
// Device data plane set-up: symmetric workspaces and NVLS multicast.
//
// Replaces the reference's transport creation (reference:
// src/transport/tcp.cc:26-92, src/transport/verbs.cc:256-304): instead of
// sockets or RDMA queue pairs, every rank allocates exportable device memory
// with the CUDA VMM API, hands the POSIX fd to every peer over the bootstrap's
// Unix sockets, and maps every peer's allocation into its own address space.
// Kernels then load and store peer memory directly over NVLink.
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "common/env.h"
#include "common/log.h"
#include "runtime/comm.h"
#include "runtime/cudrv.h"

namespace vccl {
namespace {

#define CU_TRY(call)                                                          \
  do {                                                                        \
    CUresult cu_r_ = (call);                                                  \
    if (cu_r_ != CUDA_SUCCESS) {                                              \
      VERR("%s failed: %s", #call, cuErrorText(cu_r_));                       \
      return vcclSystemError;                                                 \
    }                                                                         \
  } while (0)

#define CUDART_TRY(call)                                                      \
  do {                                                                        \
    cudaError_t rt_e_ = (call);                                               \
    if (rt_e_ != cudaSuccess) {                                               \
      VERR("%s failed: %s", #call, cudaGetErrorString(rt_e_));                \
      return vcclSystemError;                                                 \
    }                                                                         \
  } while (0)

}  // namespace

vcclResult_t mapForDevice(const DriverApi* d, CUmemGenericAllocationHandle h, size_t bytes,
                          size_t align, int device, CUdeviceptr* va) {
  CU_TRY(d->memAddressReserve(va, bytes, align, 0, 0));
  CUresult r = d->memMap(*va, bytes, 0, h, 0);
  if (r != CUDA_SUCCESS) {
    d->memAddressFree(*va, bytes);
    *va = 0;
    VERR("cuMemMap failed: %s", cuErrorText(r));
    return vcclSystemError;
  }
  CUmemAccessDesc acc;
  memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = d->memSetAccess(*va, bytes, &acc, 1);
  if (r != CUDA_SUCCESS) {
    d->memUnmap(*va, bytes);
    d->memAddressFree(*va, bytes);
    *va = 0;
    VERR("cuMemSetAccess failed: %s", cuErrorText(r));
    return vcclSystemError;
  }
  return vcclSuccess;
}

namespace {

size_t roundUp(size_t x, size_t a) { return (x + a - 1) / a * a; }

CUmemAllocationProp exportableProp(int device) {
  CUmemAllocationProp prop;
  memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return prop;
}

// Allocate `bytes` (already rounded) on this device, export, exchange, map
// every rank's allocation.
vcclResult_t symmetricAlloc(Bootstrap* bs, DeviceState* ds, size_t bytes, size_t align,
                            SymmetricBuffer* b) {
  const DriverApi* d = driverApi();
  const int n = bs->nranks(), me = bs->rank();
  CUmemAllocationProp prop = exportableProp(ds->device);
  b->bytes = bytes;
  b->align = align;
  CU_TRY(d->memCreate(&b->localHandle, bytes, &prop, 0));
  int fd = -1;
  CU_TRY(d->memExport(&fd, b->localHandle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0));
  std::vector<std::vector<int>> fds;
  vcclResult_t res = bs->exchangeFds({fd}, &fds);
  closeFd(fd);
  VTRY(res);
  b->handles.assign(n, 0);
  b->va.assign(n, 0);
  for (int p = 0; p < n; p++) {
    if (p == me) {
      b->handles[p] = b->localHandle;
    } else if (res == vcclSuccess) {
      CUresult r = d->memImport(&b->handles[p],
                                reinterpret_cast<void*>(static_cast<uintptr_t>(fds[p][0])),
                                CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
      if (r != CUDA_SUCCESS) {
        VERR("cuMemImportFromShareableHandle (rank %d) failed: %s", p, cuErrorText(r));
        res = vcclSystemError;
      }
    }
    for (int f : fds[p]) closeFd(f);
  }
  VTRY(res);
  for (int p = 0; p < n; p++) VTRY(mapForDevice(d, b->handles[p], bytes, align, ds->device, &b->va[p]));
  return vcclSuccess;
}

void symmetricFree(const DriverApi* d, int me, SymmetricBuffer* b) {
  for (size_t p = 0; p < b->va.size(); p++) {
    if (b->va[p]) {
      d->memUnmap(b->va[p], b->bytes);
      d->memAddressFree(b->va[p], b->bytes);
    }
    if (b->handles.size() > p && b->handles[p] && static_cast<int>(p) != me) d->memRelease(b->handles[p]);
  }
  if (b->localHandle) d->memRelease(b->localHandle);
  b->va.clear();
  b->handles.clear();
  b->localHandle = 0;
}

void multicastTeardown(const DriverApi* d, DeviceState* ds) {
  SymmetricBuffer& b = ds->data;
  if (b.mcVa) {
    d->memUnmap(b.mcVa, b.bytes);
    d->memAddressFree(b.mcVa, b.bytes);
    b.mcVa = 0;
  }
  if (b.mcBound) {
    d->mcUnbind(b.mcHandle, ds->cuDevice, 0, b.bytes);
    b.mcBound = false;
  }
  if (b.mcHandle) {
    d->memRelease(b.mcHandle);
    b.mcHandle = 0;
  }
}

vcclResult_t multicastSetup(Bootstrap* bs, DeviceState* ds) {
  const DriverApi* d = driverApi();
  SymmetricBuffer& b = ds->data;
  const int n = bs->nranks(), me = bs->rank();
  CUmulticastObjectProp mp;
  memset(&mp, 0, sizeof(mp));
  mp.numDevices = static_cast<unsigned int>(n);
  mp.size = b.bytes;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  bool ok = true;
  int fd = -1;
  if (me == 0) {
    ok = d->mcCreate(&b.mcHandle, &mp) == CUDA_SUCCESS &&
         d->memExport(&fd, b.mcHandle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) == CUDA_SUCCESS;
  }
  if (!everyone(bs, ok)) {
    closeFd(fd);
    multicastTeardown(d, ds);
    return vcclInternalError;
  }
  std::vector<int> fds;
  if (me == 0) fds.push_back(fd);
  VTRY(bs->broadcastFds(0, &fds, 1));
  if (me == 0) {
    closeFd(fd);
  } else {
    ok = fds.size() == 1 &&
         d->memImport(&b.mcHandle, reinterpret_cast<void*>(static_cast<uintptr_t>(fds[0])),
                      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
    for (int f : fds) closeFd(f);
  }
  ok = ok && d->mcAddDevice(b.mcHandle, ds->cuDevice) == CUDA_SUCCESS;
  // Every device must be added before any memory is bound.
  if (!everyone(bs, ok)) {
    multicastTeardown(d, ds);
    return vcclInternalError;
  }
  CUresult br = d->mcBindMem(b.mcHandle, 0, b.localHandle, 0, b.bytes, 0);
  ok = br == CUDA_SUCCESS;
  if (!ok) VWARN("cuMulticastBindMem failed: %s", cuErrorText(br));
  b.mcBound = ok;
  if (!everyone(bs, ok)) {
    multicastTeardown(d, ds);
    return vcclInternalError;
  }
  ok = mapForDevice(d, b.mcHandle, b.bytes, b.align, ds->device, &b.mcVa) == vcclSuccess;
  if (!everyone(bs, ok)) {
    multicastTeardown(d, ds);
    return vcclInternalError;
  }
  return vcclSuccess;
}

}  // namespace

vcclResult_t deviceStateCreate(Bootstrap* bs, int device, std::unique_ptr<DeviceState>* out) {
  const DriverApi* d = driverApi();
  if (d == nullptr) return vcclSystemError;
  auto ds = std::make_unique<DeviceState>();
  ds->device = device;
  CUDART_TRY(cudaSetDevice(device));
  CUDART_TRY(cudaFree(nullptr));
  CU_TRY(d->deviceGet(&ds->cuDevice, device));
  CUDART_TRY(cudaDeviceGetAttribute(&ds->smCount, cudaDevAttrMultiProcessorCount, device));
  CUDART_TRY(cudaStreamCreateWithFlags(&ds->stream, cudaStreamNonBlocking));
  CUDART_TRY(cudaHostAlloc(reinterpret_cast<void**>(&ds->hostStatus), 64,
                           cudaHostAllocMapped | cudaHostAllocPortable));
  CUDART_TRY(cudaHostAlloc(reinterpret_cast<void**>(&ds->hostAbort), 64,
                           cudaHostAllocMapped | cudaHostAllocPortable));
  memset(ds->hostStatus, 0, 64);
  memset(ds->hostAbort, 0, 64);
  CUDART_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&ds->devStatus), ds->hostStatus, 0));
  CUDART_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&ds->devAbort), ds->hostAbort, 0));

  const int n = bs->nranks(), me = bs->rank();
  ds->nblocks = static_cast<int>(envLong("VCCL_NBLOCKS", 64));
  if (ds->nblocks < 1) ds->nblocks = 1;
  if (ds->nblocks > dev::kMaxBlocks) ds->nblocks = dev::kMaxBlocks;
  // One-hop LL sends (n-1) x 2 x payload from every rank, so its useful range
  // shrinks with the rank count.
  const size_t llDefault = n <= 2 ? (1u << 20) : n <= 4 ? (512u << 10) : (256u << 10);
  // The reference's latency/bandwidth crossover of all-reduce
  // (VCCL_ALLREDUCE_RD_MAX) is the fallback name of the same threshold.
  ds->llMaxBytes = envBytes("VCCL_LL_MAX", envBytes("VCCL_ALLREDUCE_RD_MAX", llDefault));
  if (ds->llMaxBytes > dev::kLLMaxBytes) ds->llMaxBytes = dev::kLLMaxBytes;
  ds->ll2MaxBytes = envBytes("VCCL_LL2_MAX", 4u << 20);
  // Pipelined NVLS all-reduce from 256 MiB: measured on 8 B200 (bf16, bus
  // GB/s) 611.6 vs 591.4 for the staged NVLS kernel at 256 MiB and 632.2 vs
  // 544.6 at 1 GiB, but 436.2 vs 504.2 at 64 MiB.  VCCL_NVLS_PIPE_MIN=<bytes>
  // moves the threshold (0: never); VCCL_ALLREDUCE_ALGO=nvls_pipe or a tuning
  // rule picks it per call.
  ds->nvlsMinRanks = static_cast<int>(envLong("VCCL_NVLS_MIN_RANKS", 4));
  ds->nvlsMinBytes = envBytes("VCCL_NVLS_MIN", 512u << 10);
  ds->nvlsPipeMin = envBytes("VCCL_NVLS_PIPE_MIN", 256u << 20);
  ds->nvlsPieces = static_cast<int>(envLong("VCCL_NVLS_PIECES", 4));
  ds->windowsEnabled = envLong("VCCL_WINDOW", 1) != 0;
  // Windows on demand for plain device buffers (off unless asked for).
  ds->regCacheOn = ds->windowsEnabled && envLong("VCCL_REG_CACHE", 0) != 0 && envLong("VCCL_MR_CACHE", 1) != 0;
  // Each consulting call costs one bootstrap allgather (measured on a CPU
  // host over loopback TCP: about 40 / 77 / 122 us at 2 / 4 / 8 ranks), so
  // only large messages, whose staging copies cost more, consult the cache.
  ds->regCacheMin = envBytes("VCCL_REG_CACHE_MIN", 64u << 20);
  // Capacity: the reference's VCCL_MR_CACHE (LRU entries, default 16) is
  // honoured as the fallback name.
  ds->regCacheEntries = regCacheCapacityFromEnv();
  ds->orderLaunches = envLong("VCCL_LAUNCH_ORDER", 1) != 0;
  // Per GPU, the switch moves about S each way for a window all-reduce of
  // S bytes against 2 (n-1)/n S for the point-to-point kernel.
  ds->windowNvlsMinRanks = static_cast<int>(envLong("VCCL_WINDOW_NVLS_MIN_RANKS", 3));
  if (ds->nvlsPieces < 1) ds->nvlsPieces = 1;
  // An LL all-gather moves the same (n-1) x 2 x payload as the one-shot LL
  // all-reduce and needs no barrier.  At 8 ranks with 1 MiB per rank the LL
  // all-reduce (same traffic) took 33 us where the pull all-gather took
  // 73 us, so all-gather stays on LL up to the LL slot size.
  // Per-rank payload up to which all-gather takes the LL kernel; the
  // reference's name for its latency/bandwidth crossover is accepted too.
  ds->llAgMaxBytes = envBytes("VCCL_LL_AG_MAX", envBytes("VCCL_ALLGATHER_RD_MAX", dev::kLLMaxBytes));
  {
    const std::string tf = envStr("VCCL_TUNING_FILE", "");
    if (!tf.empty()) ds->tuning = loadTuningFile(tf.c_str());
  }
  if (ds->llAgMaxBytes > dev::kLLMaxBytes) ds->llAgMaxBytes = dev::kLLMaxBytes;
  // LL epochs are per block, so every rank must launch the same LL grid; the
  // fused LL kernels run in clusters of 8, hence the multiple of 8.
  long llb = envLong("VCCL_LL_BLOCKS", dev::kLLBlocks);
  llb = llb < 8 ? 8 : llb > dev::kMaxLLBlocks ? dev::kMaxLLBlocks : llb;
  ds->llBlocks = static_cast<int>(llb / 8 * 8);
  // Every rank must pick the same path for a fused call, so this is agreed
  // on below with the workspace sizes.
  ds->fusedSmallRows = static_cast<int>(envLong("VCCL_FUSED_SMALL_M", 512));

  if (n > 1) {
    if (n > dev::kMaxRanks) {
      VERR("device communicators support at most %d ranks (one NVSwitch domain)", dev::kMaxRanks);
      return vcclInvalidUsage;
    }
    // Granularities: every rank computes the same values on identical GPUs;
    // the allgather below double-checks the resulting sizes.
    CUmemAllocationProp prop = exportableProp(device);
    size_t gran = 0;
    CU_TRY(d->memGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
    size_t dataAlign = gran;
    ds->gran = gran;
    const bool tryNvls = envLong("VCCL_NVLS_ENABLE", 1) != 0 && d->mcCreate != nullptr;
    int mcCap = 0;
    if (tryNvls) d->deviceGetAttribute(&mcCap, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, ds->cuDevice);
    size_t dataBytes = envBytes("VCCL_BUFFSIZE", 256u << 20);
    if (dataBytes < (4u << 20)) dataBytes = 4u << 20;
    if (mcCap) {
      CUmulticastObjectProp mp;
      memset(&mp, 0, sizeof(mp));
      mp.numDevices = static_cast<unsigned int>(n);
      mp.size = dataBytes;
      mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
      size_t mg = 0;
      if (d->mcGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED) == CUDA_SUCCESS && mg > 0)
        dataAlign = std::max(dataAlign, mg);
      else
        mcCap = 0;
    }
    dataBytes = roundUp(dataBytes, dataAlign);
    size_t fusedBytes = roundUp(envBytes("VCCL_FUSED_BUFFSIZE", 512u << 20), gran);
    // Debug layout (VCCL_GUARDS=1): every region gets a guard of at least
    // 1 MiB past the bytes the kernels use, filled with a pattern that
    // vcclxCheckGuards verifies, so a kernel writing past its region's end
    // shows up as an error code instead of silent corruption.
    const size_t guard = envLong("VCCL_GUARDS", 0) != 0 ? (1u << 20) : 0;
    const size_t ctrlUsable = guard ? dev::kCtrlBytes : roundUp(dev::kCtrlBytes, gran);
    const size_t dataUsable = dataBytes, fusedUsable = fusedBytes;
    const size_t ctrlBytes = roundUp(ctrlUsable + guard, gran);
    dataBytes = roundUp(dataUsable + guard, dataAlign);
    fusedBytes = roundUp(fusedUsable + guard, gran);
    // Every rank must choose the same algorithm and grid for a call: the
    // tuning table and every setting that steers the choice take part in the
    // agreement through a hash.
    uint64_t tuneHash = 1469598103934665603ull;
    auto mix = [&](const std::string& line) {
      for (unsigned char ch : line) tuneHash = (tuneHash ^ ch) * 1099511628211ull;
      tuneHash = (tuneHash ^ '\n') * 1099511628211ull;
    };
    for (const TuningRule& r : ds->tuning)
      mix(r.op + " " + std::to_string(r.nranks) + " " + std::to_string(r.maxBytes) + " " + r.algo);
    mix("nblocks " + std::to_string(ds->nblocks) + " ll " + std::to_string(ds->llMaxBytes) + " ll2 " +
        std::to_string(ds->ll2MaxBytes) + " llag " + std::to_string(ds->llAgMaxBytes) + " nvls " +
        std::to_string(ds->nvlsMinRanks) + " " + std::to_string(ds->nvlsMinBytes) + " pipe " +
        std::to_string(ds->nvlsPipeMin) + " " + std::to_string(ds->nvlsPieces) + " win " +
        std::to_string(ds->windowsEnabled ? 1 : 0) + " " + std::to_string(ds->windowNvlsMinRanks) + " regcache " +
        std::to_string(ds->regCacheOn ? 1 : 0) + " " + std::to_string(ds->regCacheMin) + " " +
        std::to_string(ds->regCacheEntries));
    struct Sizes { uint64_t ctrl, data, fused, llBlocks, smallRows, tuning; } mine{
        ctrlBytes, dataBytes, fusedBytes, static_cast<uint64_t>(ds->llBlocks),
        static_cast<uint64_t>(static_cast<int64_t>(ds->fusedSmallRows)), tuneHash};
    std::vector<Sizes> all(n);
    all[me] = mine;
    VTRY(bs->allGather(all.data(), sizeof(Sizes)));
    for (const Sizes& s : all) {
      if (s.ctrl != mine.ctrl || s.data != mine.data || s.fused != mine.fused || s.llBlocks != mine.llBlocks ||
          s.smallRows != mine.smallRows || s.tuning != mine.tuning) {
        VERR("ranks disagree on workspace sizes or algorithm settings (check VCCL_BUFFSIZE, VCCL_FUSED_BUFFSIZE, "
             "VCCL_GUARDS, VCCL_LL_BLOCKS, VCCL_NBLOCKS, VCCL_FUSED_SMALL_M, the VCCL_LL_* / VCCL_NVLS_* / "
             "VCCL_WINDOW* thresholds, VCCL_REG_CACHE* and VCCL_TUNING_FILE on every rank)");
        return vcclInvalidUsage;
      }
    }
    VTRY(symmetricAlloc(bs, ds.get(), ctrlBytes, gran, &ds->ctrl));
    VTRY(symmetricAlloc(bs, ds.get(), dataBytes, dataAlign, &ds->data));
    VTRY(symmetricAlloc(bs, ds.get(), fusedBytes, gran, &ds->fused));
    ds->ctrl.usable = ctrlUsable;
    ds->data.usable = dataUsable;
    ds->fused.usable = fusedUsable;
    for (SymmetricBuffer* b : {&ds->ctrl, &ds->data, &ds->fused}) {
      if (guard && b->bytes > b->usable)
        CUDART_TRY(cudaMemset(reinterpret_cast<char*>(b->va[me]) + b->usable, dev::kGuardByte,
                              b->bytes - b->usable));
    }
    CUDART_TRY(cudaMemset(reinterpret_cast<void*>(ds->ctrl.va[me]), 0, dev::kCtrlHeader));
    // LL lines start with flag 0, an epoch no LL launch ever uses.
    CUDART_TRY(cudaMemset(reinterpret_cast<void*>(ds->ctrl.va[me] + dev::kLLOff), 0, 2 * dev::kLLBytes));
    CUDART_TRY(cudaDeviceSynchronize());
    VTRY(bs->barrier());
    if (everyone(bs, mcCap != 0)) ds->nvls = multicastSetup(bs, ds.get()) == vcclSuccess;
    VINFO("rank %d/%d on device %d: workspace ctrl %zu MiB, data %zu MiB, NVLS %s", me, n, device,
          ctrlBytes >> 20, dataBytes >> 20, ds->nvls ? "on" : "off");
  }

  if (envLong("VCCL_FUSED_TRACE", 0) != 0) {
    const size_t tb = static_cast<size_t>(dev::kMaxFusedCtas) * dev::kFusedTraceSlots * 8;
    CUDART_TRY(cudaMalloc(reinterpret_cast<void**>(&ds->fusedTrace), tb));
    CUDART_TRY(cudaMemset(ds->fusedTrace, 0, tb));
  }

  dev::DevComm& dc = ds->dc;
  memset(&dc, 0, sizeof(dc));
  dc.rank = me;
  dc.nranks = n;
  for (int p = 0; p < n && n > 1; p++) {
    dc.ctrl[p] = reinterpret_cast<char*>(ds->ctrl.va[p]);
    dc.data[p] = reinterpret_cast<char*>(ds->data.va[p]);
    dc.fused[p] = reinterpret_cast<char*>(ds->fused.va[p]);
  }
  dc.fusedBytes = ds->fused.usable ? ds->fused.usable : ds->fused.bytes;
  dc.mcData = ds->nvls ? reinterpret_cast<char*>(ds->data.mcVa) : nullptr;
  dc.dataBytes = ds->data.usable ? ds->data.usable : ds->data.bytes;
  dc.status = ds->devStatus;
  dc.abortWord = ds->devAbort;
  dc.timeoutNs = deviceTimeoutNs();
  *out = std::move(ds);
  return vcclSuccess;
}

vcclResult_t deviceStateEnsureMoe(DeviceState* ds, Bootstrap* bs, size_t bytes) {
  if (ds->dc.moeBytes >= bytes) return vcclSuccess;
  cudaSetDevice(ds->device);
  const size_t want = std::max(bytes, envBytes("VCCL_MOE_BUFFSIZE", 256u << 20));
  const int n = bs->nranks(), me = bs->rank();
  if (n == 1) {
    void* p = nullptr;
    CUDART_TRY(cudaMalloc(&p, want));
    if (ds->moeLocal) cudaFree(ds->moeLocal);
    ds->moeLocal = p;
    ds->dc.moe[0] = static_cast<char*>(p);
    ds->dc.moeBytes = want;
    return vcclSuccess;
  }
  const size_t size = roundUp(want, ds->gran);
  std::vector<uint64_t> all(n);
  all[me] = size;
  VTRY(bs->allGather(all.data(), sizeof(uint64_t)));
  for (uint64_t v : all) {
    if (v != size) {
      VERR("ranks disagree on the MoE region size (capacity, hidden size and VCCL_MOE_BUFFSIZE must match)");
      return vcclInvalidUsage;
    }
  }
  if (ds->moe.bytes) {
    // Growing: every rank finishes its work in the old region first.
    CUDART_TRY(cudaDeviceSynchronize());
    VTRY(bs->barrier());
    symmetricFree(driverApi(), me, &ds->moe);
  }
  VTRY(symmetricAlloc(bs, ds, size, ds->gran, &ds->moe));
  for (int p = 0; p < n; p++) ds->dc.moe[p] = reinterpret_cast<char*>(ds->moe.va[p]);
  ds->dc.moeBytes = size;
  VINFO("rank %d: MoE region %zu MiB", me, size >> 20);
  return vcclSuccess;
}

bool devicePointers(int device, std::initializer_list<const void*> ptrs, const char* what) {
  static const bool check = envLong("VCCL_CHECK_POINTERS", 1) != 0;
  if (!check) return true;
  // Pointers that passed recently, per host thread: a decode loop passes the
  // same buffers every step, so steady-state calls query the runtime for none
  // of them.  Direct-mapped on the pointer value; an entry records the device.
  struct Seen {
    const void* p;
    int device;
  };
  constexpr int kSeen = 32;
  thread_local Seen seen[kSeen] = {};
  int i = 0;
  for (const void* p : ptrs) {
    const size_t slot = (reinterpret_cast<uintptr_t>(p) >> 8) % kSeen;
    if (p != nullptr && seen[slot].p == p && seen[slot].device == device) {
      i++;
      continue;
    }
    cudaPointerAttributes at;
    bool ok = p != nullptr && cudaPointerGetAttributes(&at, p) == cudaSuccess &&
              ((at.type == cudaMemoryTypeDevice && at.device == device) ||
               at.type == cudaMemoryTypeManaged);  // managed memory is reachable from every device
    if (ok) seen[slot] = {p, device};
    if (!ok) {
      cudaGetLastError();
      VERR("%s: pointer argument %d is not device memory of CUDA device %d", what, i, device);
      return false;
    }
    i++;
  }
  return true;
}

OrderedLaunch::OrderedLaunch(DeviceState* ds, cudaStream_t s) : ds_(ds), s_(s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (ds == nullptr || !ds->orderLaunches) return;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
    cudaGetLastError();  // e.g. the legacy stream while another stream captures
    return;
  }
  if (cs != cudaStreamCaptureStatusNone) return;
  eager_ = true;
  const LaunchOrder& o = ds->order;
  if (o.valid && o.stream != s && cudaStreamWaitEvent(s, o.ev, 0) != cudaSuccess) cudaGetLastError();
}

OrderedLaunch::~OrderedLaunch() {
  if (!eager_) return;
  LaunchOrder& o = ds_->order;
  if (o.ev == nullptr && cudaEventCreateWithFlags(&o.ev, cudaEventDisableTiming) != cudaSuccess) {
    o.ev = nullptr;
    o.valid = false;
    cudaGetLastError();
    return;
  }
  if (cudaEventRecord(o.ev, s_) == cudaSuccess) {
    o.stream = s_;
    o.valid = true;
  } else {
    o.valid = false;
    cudaGetLastError();
  }
}

void deviceStateDestroy(DeviceState* ds, Bootstrap* bs, bool peersAlive) {
  if (ds == nullptr) return;
  const DriverApi* d = driverApi();
  cudaSetDevice(ds->device);
  if (ds->stream) cudaStreamSynchronize(ds->stream);
  cudaDeviceSynchronize();
  cudaGetLastError();
  // Peers may still be reading our memory until they are done too.
  if (peersAlive && bs && bs->nranks() > 1) bs->barrier();
  if (d) {
    multicastTeardown(d, ds);
    symmetricFree(d, bs ? bs->rank() : 0, &ds->data);
    symmetricFree(d, bs ? bs->rank() : 0, &ds->fused);
    symmetricFree(d, bs ? bs->rank() : 0, &ds->moe);
    symmetricFree(d, bs ? bs->rank() : 0, &ds->ctrl);
  }
  if (ds->moeLocal) cudaFree(ds->moeLocal);
  ds->moeLocal = nullptr;
  if (ds->fusedTrace) cudaFree(ds->fusedTrace);
  ds->fusedTrace = nullptr;
  if (ds->hostStatus) cudaFreeHost(ds->hostStatus);
  if (ds->hostAbort) cudaFreeHost(ds->hostAbort);
  if (ds->stream) cudaStreamDestroy(ds->stream);
  if (ds->order.ev) cudaEventDestroy(ds->order.ev);
  ds->order = LaunchOrder{};
  ds->hostStatus = ds->hostAbort = nullptr;
  ds->stream = nullptr;
}

}  // namespace vccl
