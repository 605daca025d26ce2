// SPDX-License-Identifier: Apache-2.0
// Communicator lifecycle, ops table, memory and registration entry points.
//
// API behaviour follows the reference (reference: src/core/comm.cc:36-348):
// InitRankConfig validates its config, InitAll forms one communicator per
// device in one process, Split orders members by (key, parent rank) with
// NOCOLOR ranks taking part in the exchange and receiving NULL, Abort marks
// the communicator dead and unblocks waiters, PreMulSum scalars are
// host-immediate floats decoded from the op's datatype with freed slots
// reused, MemFree rejects unknown pointers.
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <thread>

#include "common/env.h"
#include "common/log.h"
#include "kernels/coll_abi.cuh"
#include "runtime/comm.h"
#include "runtime/cudrv.h"

using vccl::Bootstrap;

void vcclComm::noteError(vcclResult_t r) {
  if (r == vcclSuccess) return;
  vcclResult_t expect = vcclSuccess;
  asyncError.compare_exchange_strong(expect, r);
  if (r == vcclSystemError || r == vcclRemoteError || r == vcclInternalError ||
      r == vcclUnhandledError)
    aborted.store(true);
  const char* msg = vccl::threadLastError();
  if (msg && *msg) {
    std::lock_guard<std::mutex> g(errMu);
    lastError = msg;
  }
}

vcclResult_t vcclComm::pollDeviceStatus() {
  if (!dev || dev->hostStatus == nullptr) return vcclSuccess;
  volatile uint32_t* s = dev->hostStatus;
  uint32_t code = s[0];
  if (code == vccl::dev::kOk) return vcclSuccess;
  static const char* const kWhere[] = {"?", "start barrier", "LL wait", "push barrier",
                                       "reduce barrier", "NVLS barrier", "gather barrier",
                                       "send slot wait", "recv data wait", "fused kernel wait",
                                       "MoE dispatch/combine", "window collective"};
  uint32_t where = s[1];
  const char* w = where < sizeof(kWhere) / sizeof(kWhere[0]) ? kWhere[where] : "?";
  if (code == vccl::dev::kErrAborted) {
    VERR("rank %d: kernel stopped by vcclCommAbort (%s)", rank, w);
    return vcclUnhandledError;
  }
  if (code == vccl::dev::kErrTimeout) {
    VERR("rank %d: device wait timed out (%s, peer slot %u); a peer is dead or stuck "
         "(VCCL_TIMEOUT=%ds)", rank, w, s[3], vccl::watchdogSeconds());
    return vcclSystemError;
  }
  if (code == vccl::dev::kErrCapacity) {
    VERR("rank %d: MoE dispatch received more rows than its capacity (%u rows routed here); rows past the "
         "capacity were dropped", rank, s[3]);
    return vcclInvalidUsage;
  }
  if (code == vccl::dev::kErrBadArg && where == vccl::dev::kWhereWindow) {
    VERR("rank %d: a collective on registered windows was called with different offsets or counts on "
         "different ranks (block %u); nothing was transferred", rank, s[3]);
    return vcclInvalidUsage;
  }
  VERR("rank %d: kernel reported error %u (%s)", rank, code, w);
  return vcclInternalError;
}

bool vcclComm::premulScalar(vcclRedOp_t op, double* scalar) {
  std::lock_guard<std::mutex> g(opsMu);
  if (op < vcclNumOps) return false;
  size_t i = static_cast<size_t>(op) - vcclNumOps;
  if (i >= customOps.size() || !customOps[i].live) return false;
  *scalar = customOps[i].scalar;
  return true;
}

namespace {

std::mutex gAllocMu;
struct Alloc {
  size_t bytes;
  bool device;
  int dev;
  CUmemGenericAllocationHandle handle;
};
std::map<void*, Alloc> gAllocs;

}  // namespace

namespace vccl {
bool findDeviceAllocation(const void* p, size_t bytes, void** base, size_t* allocBytes,
                          CUmemGenericAllocationHandle* handle) {
  std::lock_guard<std::mutex> g(gAllocMu);
  auto it = gAllocs.upper_bound(const_cast<void*>(p));
  if (it == gAllocs.begin()) return false;
  --it;
  const char* b = static_cast<const char*>(it->first);
  const char* q = static_cast<const char*>(p);
  if (!it->second.device || q < b || q + bytes > b + it->second.bytes) return false;
  *base = it->first;
  *allocBytes = it->second.bytes;
  *handle = it->second.handle;
  return true;
}
}  // namespace vccl

void vcclComm::noteCall(const char* op, const char* algo, size_t bytes) {
  if (!profOn) return;
  std::lock_guard<std::mutex> g(profMu);
  auto& e = prof[{op, algo}];
  e.first += 1;
  e.second += bytes;
}

namespace {

std::string profText(vcclComm_t comm) {
  std::lock_guard<std::mutex> g(comm->profMu);
  std::string out;
  char line[256];
  for (const auto& kv : comm->prof) {
    std::snprintf(line, sizeof(line), "%s\t%s\t%llu\t%llu\n", kv.first.first.c_str(), kv.first.second.c_str(),
                  kv.second.first, kv.second.second);
    out += line;
  }
  return out;
}

}  // namespace

const vccl::Window* vcclComm::findWindow(const void* p, size_t bytes) {
  std::lock_guard<std::mutex> g(regMu);
  const char* q = static_cast<const char*>(p);
  for (const vccl::Window* w : windows)
    if (!w->cached && q >= w->base && q + bytes <= w->base + w->bytes) return w;
  return nullptr;
}

namespace {

vcclResult_t checkConfig(const vcclConfig_t* cfg) {
  if (cfg == nullptr) return vcclSuccess;
  if (cfg->size < sizeof(size_t)) return vcclInvalidArgument;
  return vcclSuccess;
}

// Device the calling thread works on, or -1 when none is usable.
int callerDevice() {
  if (vccl::envLong("VCCL_NO_DEVICE", 0) != 0) return -1;
  const vccl::DriverApi* drv = vccl::driverApi();
  if (drv == nullptr) return -1;
  // Prefer the device of the thread's current driver context: it is what the
  // caller's own CUDA runtime (torch, a test) made current, and this
  // library's statically linked runtime keeps separate per-thread state.
  CUdevice cd = 0;
  if (drv->ctxGetDevice(&cd) == CUDA_SUCCESS) {
    cudaSetDevice(static_cast<int>(cd));
    return static_cast<int>(cd);
  }
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return d;
}

struct DeviceIdentity {
  int32_t present;
  int32_t ordinal;
  uint64_t host;
  unsigned char uuid[16];
};

vcclResult_t initRank(vcclComm_t* out, int nranks, const vcclUniqueId& id, int rank,
                      const vcclConfig_t* cfg) {
  if (out == nullptr || nranks < 1 || rank < 0 || rank >= nranks) return vcclInvalidArgument;
  *out = nullptr;
  auto c = std::make_unique<vcclComm>();
  c->regCache.setCapacity(vccl::regCacheCapacityFromEnv());
  c->profOn = vccl::envLong("VCCL_PROF", 0) != 0;
  c->rank = rank;
  c->nranks = nranks;
  if (cfg && cfg->size >= offsetof(vcclConfig_t, blocking) + sizeof(int)) c->blocking = cfg->blocking != 0;
  VTRY(Bootstrap::create(id, rank, nranks, &c->bootstrap));

  // Agree on the device data plane: either every rank has a distinct GPU on
  // one host, or the communicator has no device (host buffers, host data
  // plane).
  const int device = callerDevice();
  std::vector<DeviceIdentity> ids(nranks);
  DeviceIdentity& mine = ids[rank];
  memset(&mine, 0, sizeof(mine));
  mine.present = device >= 0;
  mine.ordinal = device;
  mine.host = vccl::hostFingerprint();
  if (device >= 0) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) memcpy(mine.uuid, &prop.uuid, 16);
  }
  VTRY(c->bootstrap->allGather(ids.data(), sizeof(DeviceIdentity)));
  int withDev = 0;
  for (const DeviceIdentity& d : ids) withDev += d.present ? 1 : 0;
  if (withDev != 0 && withDev != nranks) {
    VERR("some ranks have a CUDA device and some do not; cannot form a device communicator "
         "(VCCL_NO_DEVICE=1 on every rank moves host buffers over TCP instead)");
    return vcclInvalidUsage;
  }
  if (withDev == nranks) {
    for (int a = 0; a < nranks; a++) {
      for (int b = a + 1; b < nranks; b++) {
        if (ids[a].host != ids[b].host) {
          VERR("ranks %d and %d are on different hosts; device communicators need one NVLink domain "
               "(VCCL_NO_DEVICE=1 on every rank moves host buffers over TCP between hosts)",
               a, b);
          return vcclInvalidUsage;
        }
        if (memcmp(ids[a].uuid, ids[b].uuid, 16) == 0) {
          VERR("ranks %d and %d share one GPU; give every rank its own device", a, b);
          return vcclInvalidUsage;
        }
      }
    }
    VTRY(vccl::deviceStateCreate(c->bootstrap.get(), device, &c->dev));
  }
  VINFO("comm ready: rank %d/%d, device %d", rank, nranks, device);
  *out = c.release();
  return vcclSuccess;
}

float decodeHalf(uint16_t h) {
  const int e = (h >> 10) & 0x1f;
  const int m = h & 0x3ff;
  float v;
  if (e == 0)
    v = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31)
    v = m ? NAN : INFINITY;
  else
    v = std::ldexp(static_cast<float>(m | 0x400), e - 25);
  return (h & 0x8000) ? -v : v;
}

}  // namespace

extern "C" {

vcclResult_t vcclGetVersion(int* version) {
  if (version == nullptr) return vcclInvalidArgument;
  *version = VCCL_VERSION_CODE;
  return vcclSuccess;
}


const char* vcclGetLastError(vcclComm_t comm) {
  if (comm != nullptr) {
    std::lock_guard<std::mutex> g(comm->errMu);
    if (!comm->lastError.empty()) return comm->lastError.c_str();
  }
  return vccl::threadLastError();
}

vcclResult_t vcclGetUniqueId(vcclUniqueId* id) {
  if (id == nullptr) return vcclInvalidArgument;
  return vccl::makeUniqueId(id);
}

vcclResult_t vcclCommInitRank(vcclComm_t* comm, int nranks, vcclUniqueId id, int rank) {
  return initRank(comm, nranks, id, rank, nullptr);
}

vcclResult_t vcclCommInitRankConfig(vcclComm_t* comm, int nranks, vcclUniqueId id, int rank,
                                    vcclConfig_t* config) {
  VTRY(checkConfig(config));
  return initRank(comm, nranks, id, rank, config);
}

vcclResult_t vcclCommInitAll(vcclComm_t* comms, int ndev, const int* devlist) {
  if (comms == nullptr || ndev < 1) return vcclInvalidArgument;
  const bool useDevices = vccl::driverApi() != nullptr && vccl::envLong("VCCL_NO_DEVICE", 0) == 0;
  if (useDevices) {
    int count = 0;
    cudaGetDeviceCount(&count);
    for (int i = 0; i < ndev; i++) {
      int d = devlist ? devlist[i] : i;
      if (d < 0 || d >= count) {
        VERR("vcclCommInitAll: device %d out of range (%d visible)", d, count);
        return vcclInvalidArgument;
      }
    }
  }
  vcclUniqueId id;
  VTRY(vcclGetUniqueId(&id));
  std::vector<vcclResult_t> res(ndev, vcclSuccess);
  std::vector<std::thread> th;
  for (int i = 0; i < ndev; i++) {
    th.emplace_back([&, i] {
      if (useDevices) cudaSetDevice(devlist ? devlist[i] : i);
      res[i] = vcclCommInitRank(&comms[i], ndev, id, i);
    });
  }
  for (auto& t : th) t.join();
  for (int i = 0; i < ndev; i++)
    if (res[i] != vcclSuccess) return res[i];
  return vcclSuccess;
}

vcclResult_t vcclCommSplit(vcclComm_t comm, int color, int key, vcclComm_t* newcomm,
                           vcclConfig_t* config) {
  if (comm == nullptr || newcomm == nullptr) return vcclInvalidArgument;
  VTRY(checkConfig(config));
  if (comm->aborted.load()) return vcclInvalidUsage;
  *newcomm = nullptr;
  struct Entry { int32_t color, key; };
  std::vector<Entry> all(comm->nranks);
  all[comm->rank] = {color, key};
  VTRY(comm->bootstrap->allGather(all.data(), sizeof(Entry)));
  // New order: (key, parent rank) among ranks of my color.
  std::vector<std::pair<int32_t, int>> group;
  if (color >= 0)
    for (int r = 0; r < comm->nranks; r++)
      if (all[r].color == color) group.emplace_back(all[r].key, r);
  std::sort(group.begin(), group.end());
  int myNew = -1;
  for (size_t i = 0; i < group.size(); i++)
    if (group[i].second == comm->rank) myNew = static_cast<int>(i);
  // The first member of each group creates the id; everyone publishes.
  std::vector<vcclUniqueId> ids(comm->nranks);
  memset(ids.data(), 0, ids.size() * sizeof(vcclUniqueId));
  if (myNew == 0) VTRY(vccl::makeUniqueId(&ids[comm->rank], false));
  VTRY(comm->bootstrap->allGather(ids.data(), sizeof(vcclUniqueId)));
  if (color < 0) return vcclSuccess;
  if (comm->dev) cudaSetDevice(comm->dev->device);
  vcclConfig_t cfg = VCCL_CONFIG_INITIALIZER;
  cfg.blocking = config ? config->blocking : (comm->blocking ? 1 : 0);
  return initRank(newcomm, static_cast<int>(group.size()), ids[group[0].second], myNew, &cfg);
}

vcclResult_t vcclCommFinalize(vcclComm_t comm) {
  if (comm == nullptr) return vcclInvalidArgument;
  if (comm->dev) {
    cudaSetDevice(comm->dev->device);
    cudaStreamSynchronize(comm->dev->stream);
    VTRY(comm->pollDeviceStatus());
  }
  return vcclSuccess;
}

vcclResult_t vcclCommAbort(vcclComm_t comm) {
  if (comm == nullptr) return vcclInvalidArgument;
  comm->aborted.store(true);
  if (comm->dev && comm->dev->hostAbort) {
    *reinterpret_cast<volatile uint32_t*>(comm->dev->hostAbort) = 1u;
  }
  vccl::setThreadLastError("communicator aborted by vcclCommAbort");
  comm->noteError(vcclUnhandledError);
  if (comm->bootstrap) comm->bootstrap->abort();
  {
    std::lock_guard<std::mutex> g(comm->hostPlaneMu);
    if (comm->hostPlane) comm->hostPlane->abort();
  }
  return vcclSuccess;
}

vcclResult_t vcclCommGetAsyncError(vcclComm_t comm, vcclResult_t* err) {
  if (comm == nullptr || err == nullptr) return vcclInvalidArgument;
  vcclResult_t dev = comm->pollDeviceStatus();
  if (dev != vcclSuccess) comm->noteError(dev);
  *err = comm->asyncError.load();
  return vcclSuccess;
}

vcclResult_t vcclCommDestroy(vcclComm_t comm) {
  if (comm == nullptr) return vcclSuccess;
  if (comm->profOn) {
    // One line per (operation, algorithm) this rank ran.
    std::string text = profText(comm);
    size_t pos = 0;
    while (pos < text.size()) {
      const size_t end = text.find('\n', pos);
      std::string row = text.substr(pos, end - pos);
      pos = end + 1;
      const size_t t1 = row.find('\t'), t2 = row.find('\t', t1 + 1), t3 = row.find('\t', t2 + 1);
      std::fprintf(stderr, "[VCCL_PROF r%d] %s, %s: %s calls, %.3f MiB\n", comm->rank, row.substr(0, t1).c_str(),
                   row.substr(t1 + 1, t2 - t1 - 1).c_str(), row.substr(t2 + 1, t3 - t2 - 1).c_str(),
                   std::strtoull(row.substr(t3 + 1).c_str(), nullptr, 10) / 1048576.0);
    }
  }
  // Cached windows hold the peers' allocations open: drop them together
  // (every rank holds the same entries) before any rank goes on to free its
  // memory.  An aborted communicator skips the meetings; its windows are
  // released locally below.
  if (comm->dev && !comm->aborted.load() && !comm->regCache.entries().empty()) (void)vccl::regCacheFlush(comm);
  {
    std::lock_guard<std::mutex> g(comm->regMu);
    const vccl::DriverApi* d = vccl::driverApi();
    for (vccl::Registration* r : comm->regs) {
      if (r->hostPinned) cudaHostUnregister(r->base);
      if (r->mapped) munmap(r->mapped, r->mappedBytes);
      if (r->extMem) cudaDestroyExternalMemory(r->extMem);
      if (r->importedVa && d) {
        d->memUnmap(r->importedVa, r->importedBytes);
        d->memAddressFree(r->importedVa, r->importedBytes);
      }
      if (r->imported && d) d->memRelease(r->imported);
      delete r;
    }
    comm->regs.clear();
    if (!comm->windows.empty() && comm->dev) {
      cudaSetDevice(comm->dev->device);
      cudaDeviceSynchronize();  // no kernel of this process still reads a peer's window
      for (vccl::Window* w : comm->windows) {
        vccl::windowRelease(comm->dev.get(), comm->rank, w);
        delete w;
      }
    }
    comm->windows.clear();
  }
  if (comm->dev) {
    vccl::deviceStateDestroy(comm->dev.get(), comm->bootstrap.get(), !comm->aborted.load());
    comm->dev.reset();
  }
  delete comm;
  return vcclSuccess;
}

extern "C" vcclResult_t vcclxProfSummary(vcclComm_t comm, char* buf, size_t len) {
  if (comm == nullptr || buf == nullptr || len == 0) return vcclInvalidArgument;
  const std::string text = profText(comm);
  const size_t n = text.size() < len - 1 ? text.size() : len - 1;
  memcpy(buf, text.data(), n);
  buf[n] = '\0';
  return text.size() < len ? vcclSuccess : vcclInvalidArgument;
}

vcclResult_t vcclCommCount(const vcclComm_t comm, int* count) {
  if (comm == nullptr || count == nullptr) return vcclInvalidArgument;
  *count = comm->nranks;
  return vcclSuccess;
}

vcclResult_t vcclCommUserRank(const vcclComm_t comm, int* rank) {
  if (comm == nullptr || rank == nullptr) return vcclInvalidArgument;
  *rank = comm->rank;
  return vcclSuccess;
}

vcclResult_t vcclCommDevice(const vcclComm_t comm, int* device) {
  if (comm == nullptr || device == nullptr) return vcclInvalidArgument;
  *device = comm->device();
  return vcclSuccess;
}

vcclResult_t vcclRedOpCreatePreMulSum(vcclRedOp_t* op, void* scalar, vcclDataType_t dt,
                                      vcclScalarResidence_t residence, vcclComm_t comm) {
  if (op == nullptr || scalar == nullptr || comm == nullptr) return vcclInvalidArgument;
  if (residence != vcclScalarHostImmediate) {
    VERR("PreMulSum: only vcclScalarHostImmediate scalars are supported");
    return vcclInvalidArgument;
  }
  double v;
  switch (dt) {
    case vcclFloat32: v = *static_cast<const float*>(scalar); break;
    case vcclFloat64: v = *static_cast<const double*>(scalar); break;
    case vcclFloat16: v = decodeHalf(*static_cast<const uint16_t*>(scalar)); break;
    case vcclBfloat16: {
      uint32_t bits = static_cast<uint32_t>(*static_cast<const uint16_t*>(scalar)) << 16;
      float f;
      memcpy(&f, &bits, 4);
      v = f;
      break;
    }
    default:
      return vcclInvalidArgument;
  }
  std::lock_guard<std::mutex> g(comm->opsMu);
  size_t slot = comm->customOps.size();
  for (size_t i = 0; i < comm->customOps.size(); i++)
    if (!comm->customOps[i].live) { slot = i; break; }
  if (slot == comm->customOps.size()) comm->customOps.push_back({});
  comm->customOps[slot] = {v, true};
  *op = static_cast<vcclRedOp_t>(vcclNumOps + slot);
  return vcclSuccess;
}

vcclResult_t vcclRedOpDestroy(vcclRedOp_t op, vcclComm_t comm) {
  if (comm == nullptr || op < vcclNumOps) return vcclInvalidArgument;
  std::lock_guard<std::mutex> g(comm->opsMu);
  size_t i = static_cast<size_t>(op) - vcclNumOps;
  if (i >= comm->customOps.size() || !comm->customOps[i].live) return vcclInvalidArgument;
  comm->customOps[i].live = false;
  return vcclSuccess;
}

vcclResult_t vcclMemAlloc(void** ptr, size_t size) {
  if (ptr == nullptr || size == 0) return vcclInvalidArgument;
  const vccl::DriverApi* d = vccl::driverApi();
  int dev = -1;
  if (d && vccl::envLong("VCCL_NO_DEVICE", 0) == 0 && cudaGetDevice(&dev) == cudaSuccess) {
    CUmemAllocationProp prop;
    memset(&prop, 0, sizeof(prop));
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = dev;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t gran = 0;
    if (d->memGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM) != CUDA_SUCCESS) return vcclSystemError;
    size_t bytes = (size + gran - 1) / gran * gran;
    CUmemGenericAllocationHandle h = 0;
    if (d->memCreate(&h, bytes, &prop, 0) != CUDA_SUCCESS) return vcclSystemError;
    CUdeviceptr va = 0;
    if (d->memAddressReserve(&va, bytes, gran, 0, 0) != CUDA_SUCCESS) {
      d->memRelease(h);
      return vcclSystemError;
    }
    CUmemAccessDesc acc;
    memset(&acc, 0, sizeof(acc));
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = dev;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    if (d->memMap(va, bytes, 0, h, 0) != CUDA_SUCCESS) {
      d->memAddressFree(va, bytes);
      d->memRelease(h);
      return vcclSystemError;
    }
    if (d->memSetAccess(va, bytes, &acc, 1) != CUDA_SUCCESS) {
      d->memUnmap(va, bytes);
      d->memAddressFree(va, bytes);
      d->memRelease(h);
      return vcclSystemError;
    }
    void* p = reinterpret_cast<void*>(va);
    std::lock_guard<std::mutex> g(gAllocMu);
    gAllocs[p] = {bytes, true, dev, h};
    *ptr = p;
    return vcclSuccess;
  }
  cudaGetLastError();
  const long page = sysconf(_SC_PAGESIZE);
  size_t bytes = (size + page - 1) / page * page;
  void* p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (p == MAP_FAILED) return vcclSystemError;
  std::lock_guard<std::mutex> g(gAllocMu);
  gAllocs[p] = {bytes, false, -1, 0};
  *ptr = p;
  return vcclSuccess;
}

vcclResult_t vcclMemFree(void* ptr) {
  if (ptr == nullptr) return vcclSuccess;
  Alloc a;
  {
    std::lock_guard<std::mutex> g(gAllocMu);
    auto it = gAllocs.find(ptr);
    if (it == gAllocs.end()) return vcclInvalidArgument;
    a = it->second;
    gAllocs.erase(it);
  }
  if (!a.device) {
    munmap(ptr, a.bytes);
    return vcclSuccess;
  }
  const vccl::DriverApi* d = vccl::driverApi();
  // Kernels still using the memory finish first (on the allocation's device,
  // which need not be the caller's current one).
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != a.dev) cudaSetDevice(a.dev);
  cudaDeviceSynchronize();
  if (cur != a.dev && cur >= 0) cudaSetDevice(cur);
  CUdeviceptr va = reinterpret_cast<CUdeviceptr>(ptr);
  d->memUnmap(va, a.bytes);
  d->memAddressFree(va, a.bytes);
  d->memRelease(a.handle);
  return vcclSuccess;
}

}  // extern "C"

namespace {
// Makes the communicator's device current for one call and gives the caller
// back its own current device afterwards.
class DeviceScope {
 public:
  explicit DeviceScope(const vcclComm* comm) {
    if (comm == nullptr || !comm->dev) return;
    if (cudaGetDevice(&prev_) != cudaSuccess) {
      cudaGetLastError();
      prev_ = -1;
    }
    if (prev_ != comm->dev->device) cudaSetDevice(comm->dev->device);
  }
  ~DeviceScope() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;

 private:
  int prev_ = -1;
};
}  // namespace

extern "C" {

vcclResult_t vcclCommRegister(vcclComm_t comm, void* buff, size_t bytes, vcclMemHandle_t* handle) {
  if (comm == nullptr || buff == nullptr || bytes == 0 || handle == nullptr) return vcclInvalidArgument;
  auto reg = std::make_unique<vccl::Registration>();
  reg->base = buff;
  reg->bytes = bytes;
  DeviceScope scope(comm);
  if (comm->dev) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, buff) == cudaSuccess && at.type == cudaMemoryTypeUnregistered) {
      // Host memory: pin it so staging copies are asynchronous DMA.
      if (cudaHostRegister(buff, bytes, cudaHostRegisterPortable) == cudaSuccess) reg->hostPinned = true;
    }
    cudaGetLastError();
  }
  std::lock_guard<std::mutex> g(comm->regMu);
  comm->regs.push_back(reg.get());
  *handle = reg.release();
  return vcclSuccess;
}

vcclResult_t vcclCommRegisterDmaBuf(vcclComm_t comm, int fd, uint64_t offset, size_t bytes, void** ptr,
                                    vcclMemHandle_t* handle) {
  if (comm == nullptr || fd < 0 || bytes == 0 || ptr == nullptr || handle == nullptr)
    return vcclInvalidArgument;
  auto reg = std::make_unique<vccl::Registration>();
  const vccl::DriverApi* d = vccl::driverApi();
  DeviceScope scope(comm);
  if (comm->dev && d) {
    // 1. A CUDA VMM export: import the allocation and map it here.
    CUmemGenericAllocationHandle h = 0;
    int dupFd = dup(fd);
    if (d->memImport(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(dupFd)),
                     CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS) {
      close(dupFd);
      size_t gran = 0;
      CUmemAllocationProp prop;
      memset(&prop, 0, sizeof(prop));
      prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
      prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
      prop.location.id = comm->dev->device;
      d->memGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM);
      size_t span = (offset + bytes + gran - 1) / gran * gran;
      CUdeviceptr va = 0;
      CUmemAccessDesc acc;
      memset(&acc, 0, sizeof(acc));
      acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
      acc.location.id = comm->dev->device;
      acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
      if (d->memAddressReserve(&va, span, gran, 0, 0) == CUDA_SUCCESS &&
          d->memMap(va, span, 0, h, 0) == CUDA_SUCCESS && d->memSetAccess(va, span, &acc, 1) == CUDA_SUCCESS) {
        reg->imported = h;
        reg->importedVa = va;
        reg->importedBytes = span;
        reg->base = reinterpret_cast<void*>(va + offset);
        reg->bytes = bytes;
      } else {
        if (va) d->memAddressFree(va, span);
        d->memRelease(h);
      }
    } else {
      close(dupFd);
    }
    // 2. An opaque fd from another API's external-memory export.
    if (reg->base == nullptr) {
      cudaExternalMemoryHandleDesc ed;
      memset(&ed, 0, sizeof(ed));
      ed.type = cudaExternalMemoryHandleTypeOpaqueFd;
      ed.handle.fd = dup(fd);  // CUDA takes ownership on success
      ed.size = offset + bytes;
      cudaExternalMemory_t em = nullptr;
      if (cudaImportExternalMemory(&em, &ed) == cudaSuccess) {
        cudaExternalMemoryBufferDesc bd;
        memset(&bd, 0, sizeof(bd));
        bd.offset = offset;
        bd.size = bytes;
        void* p = nullptr;
        if (cudaExternalMemoryGetMappedBuffer(&p, em, &bd) == cudaSuccess) {
          reg->extMem = em;
          reg->base = p;
          reg->bytes = bytes;
        } else {
          cudaDestroyExternalMemory(em);
        }
      } else {
        close(ed.handle.fd);
      }
      cudaGetLastError();
    }
  }
  // 3. A CPU-mappable dmabuf (udmabuf, memfd): map it; collectives stage it.
  if (reg->base == nullptr) {
    void* m = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, static_cast<off_t>(offset));
    if (m == MAP_FAILED) {
      VERR("vcclCommRegisterDmaBuf: fd %d is neither a CUDA export nor mappable", fd);
      return vcclSystemError;
    }
    reg->mapped = m;
    reg->mappedBytes = bytes;
    reg->base = m;
    reg->bytes = bytes;
  }
  *ptr = reg->base;
  std::lock_guard<std::mutex> g(comm->regMu);
  comm->regs.push_back(reg.get());
  *handle = reg.release();
  return vcclSuccess;
}

vcclResult_t vcclCommDeregister(vcclComm_t comm, vcclMemHandle_t handle) {
  if (comm == nullptr || handle == nullptr) return vcclInvalidArgument;
  auto* r = static_cast<vccl::Registration*>(handle);
  std::lock_guard<std::mutex> g(comm->regMu);
  auto it = std::find(comm->regs.begin(), comm->regs.end(), r);
  if (it == comm->regs.end()) return vcclInvalidArgument;
  comm->regs.erase(it);
  DeviceScope scope(comm);
  if (r->hostPinned) cudaHostUnregister(r->base);
  if (r->mapped) munmap(r->mapped, r->mappedBytes);
  if (r->extMem) cudaDestroyExternalMemory(r->extMem);
  const vccl::DriverApi* d = vccl::driverApi();
  if (r->importedVa && d) {
    cudaDeviceSynchronize();
    d->memUnmap(r->importedVa, r->importedBytes);
    d->memAddressFree(r->importedVa, r->importedBytes);
  }
  if (r->imported && d) d->memRelease(r->imported);
  delete r;
  return vcclSuccess;
}

}  // extern "C"
