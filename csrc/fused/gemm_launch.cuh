// SPDX-License-Identifier: Apache-2.0
// Launch template shared by every GEMM-based kernel (plain, SiLU*mul,
// GEMM + reduce-scatter, all-gather + GEMM).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>

#include "fused/gemm_host.h"
#include "kernels/gemm_sm100.cuh"

namespace vccl {
namespace gemm {

template <int BN, int STAGES, typename Epi, typename Hooks>
cudaError_t launchT(const CUtensorMap& ma, const CUtensorMap& mb, const GemmShape& s, const Epi& epi,
                    const Hooks& hooks, int grid, cudaStream_t st, int* flag) {
  using L = Smem<BN, STAGES, 4 * Hooks::kEpiGroups>;
  auto kern = gemmKernel<BN, STAGES, Epi, Hooks>;
  static std::atomic<unsigned long long> attrDone{0};  // one bit per device; threads of any device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attrDone.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    attrDone.fetch_or(bit, std::memory_order_release);
  }
  kern<<<grid, ctaThreads<Hooks>(), L::kBytes, st>>>(ma, mb, s, epi, hooks, flag);
  return cudaGetLastError();
}

// gridCap > 0: at most that many CTAs; gridCap < 0: exactly -gridCap CTAs
// (fused kernels count on a fixed grid); 0: one CTA per SM at most.
// splits > 1 runs split-K (only with NoHooks tile order and EpiPartialF32).
// flag: device word the kernel sets if it abandons its work (nullptr: the
// per-device flag of errorFlag()).
template <typename Epi, typename Hooks>
cudaError_t launchGemm(const void* A, const void* B, int M, int N, int K, const Epi& epi, const Hooks& hooks,
                       cudaStream_t st, int bnOverride, int gridCap, int splits = 1, int* flag = nullptr) {
  const int bn = bnOverride > 0 ? bnOverride : pickBN(M, N);
  CUtensorMap ma, mb;
  const int aRows = M >= kBM ? kBM : (M + 7) / 8 * 8;
  if (!makeMapKMajor(&ma, A, M, K, aRows) || !makeMapKMajor(&mb, B, N, K, bn)) return cudaErrorInvalidValue;
  GemmShape s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.tilesM = (M + kBM - 1) / kBM;
  s.tilesN = (N + bn - 1) / bn;
  s.splits = splits < 1 ? 1 : splits;
  s.aRows = aRows;
  if (s.splits > s.numK()) return cudaErrorInvalidValue;
  int grid = s.tilesM * s.tilesN * s.splits;
  if (gridCap < 0) {
    grid = -gridCap;
  } else {
    const int cap = gridCap > 0 ? gridCap : smCount();
    if (grid > cap) grid = cap;
  }
  if (flag == nullptr) flag = errorFlag();
  switch (bn) {
    case 256: return launchT<256, 4>(ma, mb, s, epi, hooks, grid, st, flag);
    case 128: return launchT<128, 6>(ma, mb, s, epi, hooks, grid, st, flag);
    case 64: return launchT<64, 8>(ma, mb, s, epi, hooks, grid, st, flag);
    default: return launchT<32, 8>(ma, mb, s, epi, hooks, grid, st, flag);
  }
}

}  // namespace gemm
}  // namespace vccl
