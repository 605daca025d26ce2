// SPDX-License-Identifier: Apache-2.0
// Communicator state.
//
// Mirrors the reference communicator's responsibilities (reference:
// src/core/comm.h:19-169): rank/size, bootstrap, registrations, PreMulSum op
// table, first-error latch with abort, last-error text.  The transport and
// its MR cache are replaced by DeviceState: the symmetric NVLink workspaces,
// the optional NVLS multicast mapping, a private stream and the host-mapped
// status/abort words that kernels report through.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <initializer_list>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "control/bootstrap.h"
#include "runtime/hostplane.h"
#include "runtime/regcache.h"
#include "runtime/tuning.h"
#include "kernels/device_common.cuh"
#include "vccl.h"

namespace vccl {

// One cuMem allocation per rank, exported to and mapped by every rank.
struct SymmetricBuffer {
  size_t bytes = 0;
  size_t usable = 0;  // bytes the kernels use; [usable, bytes) is a guard region (VCCL_GUARDS=1)
  size_t align = 0;
  CUmemGenericAllocationHandle localHandle = 0;
  std::vector<CUmemGenericAllocationHandle> handles;  // per rank (imported for peers)
  std::vector<CUdeviceptr> va;                         // per rank mapping in this process
  // NVLS
  CUmemGenericAllocationHandle mcHandle = 0;
  CUdeviceptr mcVa = 0;
  bool mcBound = false;
};

// Kernels of one communicator never overlap, whatever streams they are
// issued on: they share the workspaces and barrier counters, and the fused
// kernels hold every SM while they wait for the peers.  The event is
// recorded after each eager launch; a launch on another stream first waits
// for it.
struct LaunchOrder {
  cudaEvent_t ev = nullptr;
  cudaStream_t stream = nullptr;  // stream of the last eager launch
  bool valid = false;
};

struct DeviceState {
  int device = -1;
  CUdevice cuDevice = 0;
  int smCount = 0;
  cudaStream_t stream = nullptr;   // internal stream (blocking helpers)
  SymmetricBuffer ctrl;
  SymmetricBuffer data;
  SymmetricBuffer fused;           // staging owned by the fused TP kernels
  SymmetricBuffer moe;             // MoE dispatch/combine region (first use)
  void* moeLocal = nullptr;        // single-rank MoE region (plain allocation)
  size_t gran = 0;                 // VMM allocation granularity
  bool nvls = false;
  uint32_t* hostStatus = nullptr;  // pinned + mapped
  uint32_t* devStatus = nullptr;
  uint32_t* hostAbort = nullptr;
  uint32_t* devAbort = nullptr;
  dev::DevComm dc{};
  int nblocks = 32;                // grid of barrier-based kernels
  size_t llMaxBytes = 0;           // one-hop LL threshold (per-rank payload)
  size_t llAgMaxBytes = 0;         // LL threshold of all-gather (per-rank payload)
  int llBlocks = 64;               // grid of every LL kernel, a multiple of 8
  int fusedSmallRows = 512;        // fused TP calls up to this many rows run unfused
  unsigned long long* fusedTrace = nullptr;  // per-CTA event times of the fused kernels (VCCL_FUSED_TRACE=1)
  std::vector<TuningRule> tuning;  // measured algorithm table (VCCL_TUNING_FILE)
  size_t ll2MaxBytes = 0;          // two-hop LL all-reduce threshold
  int nvlsMinRanks = 4;            // NVLS all-reduce from this many ranks (VCCL_NVLS_MIN_RANKS) ...
  size_t nvlsMinBytes = 512u << 10;  // ... and this size (VCCL_NVLS_MIN)
  size_t nvlsPipeMin = 0;          // pipelined NVLS all-reduce from this size (0: only when asked for)
  int nvlsPieces = 4;              // pieces of a pipelined NVLS all-reduce
  bool windowsEnabled = true;      // zero-copy kernels for buffers in registered windows (VCCL_WINDOW)
  int windowNvlsMinRanks = 3;      // window collectives go through the switch from this many ranks
  bool regCacheOn = false;         // windows for plain device buffers on demand (VCCL_REG_CACHE)
  size_t regCacheMin = 64u << 20;  // ... for calls whose window extent is at least this (VCCL_REG_CACHE_MIN)
  int regCacheEntries = 16;        // ... at most this many at once (VCCL_REG_CACHE_ENTRIES)
  LaunchOrder order;
  bool orderLaunches = true;       // VCCL_LAUNCH_ORDER=0: the application keeps one stream per communicator
};

// Scope of one API call's launches on stream `s`: on entry `s` waits for the
// communicator's previous launch when that went to another stream, on exit
// the call's work is recorded as the new previous launch.  Streams under
// graph capture are left alone (a capture may not wait on work outside it;
// a graph orders its own nodes, and the application orders graph launches).
// Every pointer of `ptrs` is device (or managed) memory of `device`.  The
// fused entry points refuse anything else before a kernel or a TMA map would
// fault on it (VCCL_CHECK_POINTERS=0 skips the check: one
// cudaPointerGetAttributes per pointer and call).
bool devicePointers(int device, std::initializer_list<const void*> ptrs, const char* what);

class OrderedLaunch {
 public:
  OrderedLaunch(DeviceState* ds, cudaStream_t s);
  ~OrderedLaunch();
  OrderedLaunch(const OrderedLaunch&) = delete;
  OrderedLaunch& operator=(const OrderedLaunch&) = delete;

 private:
  DeviceState* ds_;
  cudaStream_t s_;
  bool eager_ = false;
};

struct CustomOp {
  double scalar = 1.0;
  bool live = false;
};

struct Registration {
  void* base = nullptr;
  size_t bytes = 0;
  bool hostPinned = false;                    // we cudaHostRegister'ed it
  void* mapped = nullptr;                     // dmabuf host mapping we own
  size_t mappedBytes = 0;
  CUmemGenericAllocationHandle imported = 0;  // VMM import we own
  CUdeviceptr importedVa = 0;
  size_t importedBytes = 0;
  cudaExternalMemory_t extMem = nullptr;      // external-memory import we own
};

// A registered window: user memory (vcclMemAlloc or cudaMalloc) that every
// rank has mapped (vcclMemAlloc memory, when the node supports NVLS, also
// bound to a multicast object), so collectives on it read and write the
// peers' buffers in place.
struct Window {
  char* base = nullptr;  // this rank's window
  size_t bytes = 0;
  std::vector<char*> peer;  // every rank's window in this address space ([rank] = base)
  std::vector<CUdeviceptr> peerVa;  // mappings of the peers' whole allocations
  std::vector<size_t> peerVaBytes;
  std::vector<CUmemGenericAllocationHandle> peerHandle;
  std::vector<void*> ipcBase;  // peers' cudaMalloc allocations opened by IPC handle (cudaMalloc windows)
  CUmemGenericAllocationHandle localHandle = 0;  // the allocation's handle (owned by vcclMemAlloc)
  size_t localOffset = 0;                        // window offset inside that allocation
  CUmemGenericAllocationHandle mcHandle = 0;
  CUdeviceptr mcVa = 0;
  size_t mcBytes = 0;
  bool mcBound = false;
  char* mc = nullptr;  // multicast address of the window, or null
  bool cached = false;  // owned by the registration cache, not by the application
};

// The vcclMemAlloc device allocation holding [p, p + bytes): its base,
// size and VMM handle.  False for anything else.
bool findDeviceAllocation(const void* p, size_t bytes, void** base, size_t* allocBytes,
                          CUmemGenericAllocationHandle* handle);
// Shared set-up steps of the symmetric workspaces (device.cc), also used by
// window registration.
struct DriverApi;
vcclResult_t mapForDevice(const DriverApi* d, CUmemGenericAllocationHandle h, size_t bytes, size_t align,
                          int device, CUdeviceptr* va);
// Release a window's multicast binding, or that and its peer mappings
// (local steps only).
void windowReleaseMulticast(DeviceState* ds, Window* w);
void windowRelease(DeviceState* ds, int me, Window* w);
// Collective window registration (vcclCommWindowRegister); `cached` marks a
// window the registration cache owns.
vcclResult_t windowRegister(vcclComm_t comm, void* buff, size_t size, int flags, bool cached, Window** out);
// Registration cache (VCCL_REG_CACHE=1), collective: every rank calls it for
// the same call, with buffers of the same sizes.  Makes sure every rank holds
// cached windows over the call's `nbuf` buffers (entries reused, registered
// or dropped by one plan all ranks compute alike) and returns them in
// out[i], or leaves every out[i] null on every rank when the call must stay
// on the staged kernels.  `eligible`: this rank's buffers are device memory
// of its own (no staged host range).
vcclResult_t regCacheWindows(vcclComm_t comm, cudaStream_t s, const void* const* ptrs, const size_t* bytes,
                             int nbuf, bool eligible, const Window** out);
// Drop every cached window (collective).
vcclResult_t regCacheFlush(vcclComm_t comm);

vcclResult_t deviceStateCreate(Bootstrap* bs, int device, std::unique_ptr<DeviceState>* out);
// Make sure the MoE region holds at least `bytes` on every rank.  Collective
// when it allocates: every rank must call it with the same size (the MoE
// entry points derive it from arguments that must agree across ranks).
vcclResult_t deviceStateEnsureMoe(DeviceState* ds, Bootstrap* bs, size_t bytes);
void deviceStateDestroy(DeviceState* ds, Bootstrap* bs, bool peersAlive);

}  // namespace vccl

struct vcclComm {
  int rank = -1;
  int nranks = 0;
  bool blocking = true;
  std::unique_ptr<vccl::Bootstrap> bootstrap;
  std::unique_ptr<vccl::DeviceState> dev;

  std::atomic<vcclResult_t> asyncError{vcclSuccess};
  std::atomic<bool> aborted{false};
  std::mutex errMu;
  std::string lastError;

  std::vector<vccl::CustomOp> customOps;
  std::mutex opsMu;

  std::mutex regMu;
  std::vector<vccl::Registration*> regs;
  std::vector<vccl::Window*> windows;  // guarded by regMu (application and cached windows)

  std::mutex regCacheMu;        // one cache step at a time
  vccl::RegCacheBook regCache;  // guarded by regCacheMu

  // Host data plane of a communicator without a device and with more than
  // one rank (runtime/hostplane.h), made on its first data call.
  std::mutex hostPlaneMu;  // guards the pointer (vcclCommAbort reads it)
  std::unique_ptr<vccl::HostPlane> hostPlane;

  // Call profile (VCCL_PROF=1): per (operation, algorithm), calls and bytes;
  // printed when the communicator is destroyed (vcclxProfSummary reads it).
  // The reference's VCCL_PROF times its verbs steps and prints them at exit
  // (reference: src/transport/verbs.cc:57-91).
  bool profOn = false;
  std::mutex profMu;
  std::map<std::pair<std::string, std::string>, std::pair<unsigned long long, unsigned long long>> prof;
  void noteCall(const char* op, const char* algo, size_t bytes);

  // The application window holding [p, p + bytes), or null (collective
  // buffer lookup).  Cached windows are not returned: a call uses one only
  // when the cache's plan for that call picked it on every rank.
  const vccl::Window* findWindow(const void* p, size_t bytes);

  int device() const { return dev ? dev->device : -1; }

  // First error wins; fatal codes latch the communicator dead so later calls
  // fail fast with vcclInvalidUsage (reference: src/core/comm.h:150-168).
  void noteError(vcclResult_t r);
  // Pull a kernel-reported failure from the host-mapped status words.
  vcclResult_t pollDeviceStatus();
  bool premulScalar(vcclRedOp_t op, double* scalar);
};
