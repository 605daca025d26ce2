// SPDX-License-Identifier: Apache-2.0
// vcclGemmBf16NoAlloc: the bf16 GEMM of vcclGemmBf16 for callers that must
// not allocate device memory.  No counterpart in the reference.
//
// vcclGemmBf16 runs decode-shaped GEMMs (few output tiles) as split-K: each
// K split writes fp32 partials to a scratch buffer that it allocates per
// stream (and reallocates when a larger shape comes), and a second kernel
// sums them into the bf16 output.  It also allocates a small per-device
// abort flag on first use.  Some callers cannot
// allow either allocation: code that runs inside a custom allocator's hook
// (allocating there re-enters the allocator), an out-of-memory handler that
// must still make progress, or a server that reserved all free device memory
// for its KV cache at start-up and keeps none for transient scratch.  This
// entry point runs the same kernels with its split-K partials in one fixed
// `static __device__` array and its abort word in a page of static host
// memory, so it allocates nothing.
//
// Limits and rules (also stated in vccl_tp.h):
//  * The split-K partials of one call must fit in kScratchBytes (8 MiB); a
//    shape whose split-K plan needs more is rejected with
//    vcclInvalidArgument and a message naming both sizes.  Shapes that do
//    not take the split-K path use no scratch at all.
//  * The first call on each device does set-up: it resolves the array's
//    device address (cudaGetSymbolAddress, with that device current), loads
//    the module that holds the array (with lazy module loading that happens
//    here, not at library load), page-locks and maps the static abort page
//    (cudaHostRegister, once per process) and configures the kernels.  Make
//    that first call at start-up, before memory is reserved and before any
//    stream capture.
//  * Nothing in the partials region needs to start at zero: every partial
//    read by the reduction was written earlier in the same call.
//  * A launch whose pipeline wait ran out abandons its tiles and sets the
//    device's abort word; a split-K reduction that then runs writes NaN
//    instead of summing stale partials.  The next call on that device
//    returns vcclInternalError and clears the word, as vcclGemmBf16 does.
//  * Calls that can overlap in time on one device (different streams or
//    host threads without ordering between them) share the one array and
//    race.  Calls on one stream are ordered and safe.
#include <cuda_runtime.h>

#include <mutex>

#include "common/log.h"
#include "fused/gemm_launch.cuh"
#include "vccl_tp.h"

namespace vccl {
namespace gemm {
namespace {

constexpr size_t kScratchBytes = 8u << 20;  // fp32 split-K partials
constexpr int kMaxDevices = 64;
constexpr int kWordStride = 16;  // ints: one 64-byte line per device

static __device__ __align__(256) unsigned char gNoAllocArena[kScratchBytes];

// Abort words, one cache line per device, in this library's own static host
// memory (nothing allocated), page-locked and mapped into every device's
// address space by the first call.
alignas(4096) int gNoAllocAbort[kMaxDevices * kWordStride];

struct DeviceSetup {
  unsigned char* arena = nullptr;  // device address of gNoAllocArena
  int* abortDev = nullptr;         // device address of this device's abort word
};

// Set-up of the current device, done once per device.  Returns false (after
// logging) if the runtime refuses.
bool setupCurrentDevice(int* devOut, DeviceSetup* out) {
  static std::mutex mu;
  static bool registered = false;
  static DeviceSetup setup[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    VERR("vcclGemmBf16NoAlloc: no usable current device (%s)", cudaGetErrorString(e));
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  DeviceSetup& s = setup[dev];
  if (s.arena == nullptr) {
    if (!registered) {
      e = cudaHostRegister(gNoAllocAbort, sizeof(gNoAllocAbort), cudaHostRegisterMapped | cudaHostRegisterPortable);
      if (e != cudaSuccess) {
        VERR("vcclGemmBf16NoAlloc: cannot map the abort page: %s", cudaGetErrorString(e));
        return false;
      }
      registered = true;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, gNoAllocArena);
    if (e != cudaSuccess || p == nullptr) {
      VERR("vcclGemmBf16NoAlloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
      return false;
    }
    void* a = nullptr;
    e = cudaHostGetDevicePointer(&a, gNoAllocAbort, 0);
    if (e != cudaSuccess || a == nullptr) {
      VERR("vcclGemmBf16NoAlloc: no device address for the abort page on device %d: %s", dev,
           cudaGetErrorString(e));
      return false;
    }
    s.abortDev = static_cast<int*>(a) + dev * kWordStride;
    s.arena = static_cast<unsigned char*>(p);
  }
  *devOut = dev;
  *out = s;
  return true;
}

// Reads and clears the abort word of `dev`: true if a launch since the last
// call abandoned its tiles.
bool takeNoAllocAbort(int dev) {
  volatile int* w = gNoAllocAbort + dev * kWordStride;
  if (*w == 0) return false;
  *w = 0;
  return true;
}

}  // namespace

// Host-side test hook: marks the abort word of `dev` as set, the state a
// launch that abandoned its tiles leaves behind.
void noAllocInjectAbort(int dev) {
  if (dev >= 0 && dev < kMaxDevices) *reinterpret_cast<volatile int*>(gNoAllocAbort + dev * kWordStride) = 1;
}

}  // namespace gemm
}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclGemmBf16NoAlloc(const void* A, const void* W, void* C, int M, int N, int K,
                                            vcclStream_t stream) {
  if (!A || !W || !C || M <= 0 || N <= 0 || K <= 0 || (N % 16) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  int dev = 0;
  gemm::DeviceSetup ds;
  if (!gemm::setupCurrentDevice(&dev, &ds)) return vcclUnhandledError;
  if (gemm::takeNoAllocAbort(dev)) {
    VERR("vcclGemmBf16NoAlloc: an earlier call on device %d abandoned its tiles (a pipeline wait ran out); its "
         "output is invalid (NaN where it was reduced)",
         dev);
    return vcclInternalError;
  }
  float* partials = reinterpret_cast<float*>(ds.arena);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The plan of vcclGemmBf16 with the same environment (VCCL_GEMM_BN,
  // VCCL_GEMM_SPLITK), so both entry points run the same GEMM.
  const int bnEnv = static_cast<int>(gemm::envLongGemm("VCCL_GEMM_BN"));
  const gemm::SplitPlan plan = gemm::planFor(M, N, K, bnEnv, true);
  cudaError_t e;
  if (plan.splits > 1) {
    const size_t elems = static_cast<size_t>(M) * N;
    const size_t need = elems * plan.splits * sizeof(float);
    if (need > gemm::kScratchBytes) {
      VERR("vcclGemmBf16NoAlloc: M=%d N=%d K=%d needs %zu bytes of split-K scratch (%d splits); the fixed "
           "scratch holds %zu bytes",
           M, N, K, need, plan.splits, gemm::kScratchBytes);
      return vcclInvalidArgument;
    }
    gemm::EpiPartialF32 epi{partials, N, elems};
    e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, st, plan.bn, 0, plan.splits, ds.abortDev);
    if (e == cudaSuccess) e = gemm::launchSplitReduce(partials, plan.splits, elems, C, st, ds.abortDev);
  } else {
    gemm::EpiStore epi{static_cast<__nv_bfloat16*>(C), N};
    e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, st, bnEnv, 0, 1, ds.abortDev);
  }
  if (e != cudaSuccess) {
    VERR("vcclGemmBf16NoAlloc: %s", cudaGetErrorString(e));
    return gemm::launchResult(e);
  }
  return vcclSuccess;
}

// Diagnostic hook (vccl_x.h): the state a launch that abandoned its tiles on
// `device` leaves behind, set from the host so tests need no device fault.
extern "C" vcclResult_t vcclxNoAllocInjectAbort(int device) {
  if (device < 0 || device >= gemm::kMaxDevices) return vcclInvalidArgument;
  gemm::noAllocInjectAbort(device);
  return vcclSuccess;
}
