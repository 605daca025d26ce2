// SPDX-License-Identifier: Apache-2.0
// vcclGemmBf16NoAlloc: the bf16 GEMM of vcclGemmBf16 for callers that must
// not allocate device memory.
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
// entry point runs the same kernels with its scratch and its abort flag in
// one fixed device array that exists from module load, so it allocates
// nothing.
//
// Limits and rules (also stated in vccl_tp.h):
//  * The split-K partials of one call must fit in kScratchBytes (8 MiB); a
//    shape whose split-K plan needs more is rejected with
//    vcclInvalidArgument and a message naming both sizes.  Shapes that do
//    not take the split-K path use no scratch at all.
//  * The first call on each device does setup: it resolves the array's
//    device address (cudaGetSymbolAddress, with that device current) and
//    configures the kernels.  Make that first call before any stream
//    capture.
//  * Nothing in the partials region needs to start at zero: every partial
//    read by the reduction was written earlier in the same call.  The abort
//    word must start at zero, which static device storage does; the kernels
//    only set it when they abandon a launch.
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
constexpr size_t kFlagBytes = 256;          // abort word (+ padding)

static __device__ __align__(256) unsigned char gNoAllocArena[kScratchBytes + kFlagBytes];

// Device address of gNoAllocArena on the current device, resolved once per
// device.  nullptr (after logging) if the runtime refuses.
unsigned char* arenaOnCurrentDevice() {
  static std::mutex mu;
  static unsigned char* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    VERR("vcclGemmBf16NoAlloc: no usable current device (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, gNoAllocArena);
    if (e != cudaSuccess || p == nullptr) {
      VERR("vcclGemmBf16NoAlloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<unsigned char*>(p);
  }
  return addr[dev];
}

}  // namespace
}  // namespace gemm
}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclGemmBf16NoAlloc(const void* A, const void* W, void* C, int M, int N, int K,
                                            vcclStream_t stream) {
  if (!A || !W || !C || M <= 0 || N <= 0 || K <= 0 || (N % 16) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  unsigned char* arena = gemm::arenaOnCurrentDevice();
  if (arena == nullptr) return vcclUnhandledError;
  float* partials = reinterpret_cast<float*>(arena);
  int* flag = reinterpret_cast<int*>(arena + gemm::kScratchBytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const gemm::SplitPlan plan = gemm::planSplitK(M, N, K);
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
    e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, st, plan.bn, 0, plan.splits, flag);
    if (e == cudaSuccess) e = gemm::launchSplitReduce(partials, plan.splits, elems, C, st);
  } else {
    gemm::EpiStore epi{static_cast<__nv_bfloat16*>(C), N};
    e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, st, 0, 0, 1, flag);
  }
  if (e != cudaSuccess) {
    VERR("vcclGemmBf16NoAlloc: %s", cudaGetErrorString(e));
    return vcclInvalidArgument;
  }
  return vcclSuccess;
}
