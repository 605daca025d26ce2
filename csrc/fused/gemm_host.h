// SPDX-License-Identifier: Apache-2.0
// Host helpers shared by the GEMM-based fused kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

#include "vccl.h"

namespace vccl {
namespace gemm {

// K-major bf16 tensor map for rows x K with a (64 x boxRows) box, 128B swizzle.
bool makeMapKMajor(CUtensorMap* map, const void* base, int rows, int K, int boxRows);
int smCount();
// Output tile width: by default the widest whose tiles fill every SM; with
// VCCL_GEMM_PICK_WAVES=1 the one with the shortest makespan (waves x width,
// with a small charge for narrow tiles), pickBNWaves.
int pickBN(int M, int N);
int pickBNWaves(int M, int N, int sms);
int* errorFlag();
// True (once) if a GEMM on the current device set its abort flag since the
// last call; reads pinned host memory, no synchronisation.
bool takeAbortFlag();

// Split-K plan for GEMMs with too few output tiles to fill the GPU (decode
// shapes): 128-wide tiles, K split so tiles x splits approaches one wave.
// splits == 1 means no split.
struct SplitPlan {
  int bn;
  int splits;
};
SplitPlan planSplitK(int M, int N, int K);
// Plan of the CTA-pair kernel for a shape: whether to use it and with how
// many K splits (fp32 partials summed by a second kernel when > 1).
struct PairPlan {
  bool use;
  int splits;
};
// Pair-kernel plan with split-K (plain GEMM and SiLU*mul only) for `pairs`
// co-resident CTA pairs: the time of ceil(units / pairs) waves of units of
// 1 / splits of a tile, plus the fp32 partials' HBM traffic, against the
// one-SM kernel's waves (gemm.cu).
PairPlan planPair(int M, int N, int K, int bnOverride, int pairs);
float* splitScratch(cudaStream_t st, size_t bytes);

// Scratch for one call on `st`: the per-stream cached buffer, or a
// stream-ordered allocation while `st` is being captured (released with
// releaseScratch after the call's launches).
struct Scratch {
  void* p = nullptr;
  bool async = false;
  cudaStream_t st = nullptr;
  // Split-K fix-up semaphores (zero between calls), when the in-kernel
  // reduction is enabled: per stream, or a stream-ordered zeroed
  // allocation while `st` is being captured.
  uint32_t* sems = nullptr;
  bool semsAsync = false;
};
bool acquireScratch(cudaStream_t st, size_t bytes, Scratch* out);
void releaseScratch(const Scratch& s);

// In-kernel split-K reduction (EpiSplitFixup) for GEMMs of at most
// kFixupMaxRows rows, when VCCL_GEMM_SPLIT_FIXUP=1; semaphores for up to
// kSemSlots / 4 output tiles.
constexpr int kFixupMaxRows = 8;
constexpr int kSemSlots = 4096;
bool splitFixupEnabled();

// Split-K (or not) plan honouring VCCL_GEMM_BN / VCCL_GEMM_SPLITK.
SplitPlan planFor(int M, int N, int K, int bnOverride, bool allowSplit);
// fp32 scratch gemmAuto needs for this shape (0 without split-K).
size_t gemmAutoScratchBytes(int M, int N, int K, int bnOverride, bool allowSplit);
// C = A W^T (bf16), or silu(gate) * up with C of N/2 columns, split-K for
// decode shapes; ws must hold gemmAutoScratchBytes bytes when that is > 0.
// With `sems` (Scratch::sems) small split-K GEMMs reduce inside the kernel.
cudaError_t gemmAuto(const void* A, const void* W, void* C, int M, int N, int K, bool siluMul, cudaStream_t st,
                     int bnOverride, bool allowSplit, float* ws, uint32_t* sems = nullptr);
cudaError_t launchSplitReduceSilu(const float* ws, int splits, int M, int N, void* out, cudaStream_t st);

// out[i] = bf16(sum over s < splits of ws[s * elems + i]); elems % 4 == 0.
// With abortWord (a word the GEMM sets when it abandons its tiles) set when
// the reduction runs, out is filled with NaN instead.
cudaError_t launchSplitReduce(const float* ws, int splits, size_t elems, void* out, cudaStream_t st,
                              const volatile int* abortWord = nullptr);

// The GEMM of vcclGemmBf16 / vcclGemmSiluMul (split-K with per-stream
// scratch for decode shapes, CTA pairs for large ones, one-SM tiles
// otherwise), as a vccl result; `what` names the caller in error messages.
vcclResult_t gemmWithScratch(const char* what, const void* A, const void* W, void* C, int M, int N, int K,
                             bool siluMul, cudaStream_t st);

// The result code of a failed GEMM launch: vcclInvalidArgument when the
// arguments could not be described to the hardware (a tensor map the driver
// refused, a split the shape cannot take: cudaErrorInvalidValue), otherwise
// vcclUnhandledError (a launch or runtime failure, not the caller's mistake).
inline vcclResult_t launchResult(cudaError_t e) {
  return e == cudaErrorInvalidValue ? vcclInvalidArgument : vcclUnhandledError;
}

inline long envLongGemm(const char* name) {
  const char* v = std::getenv(name);
  return v ? std::strtol(v, nullptr, 10) : 0;
}

}  // namespace gemm
}  // namespace vccl
