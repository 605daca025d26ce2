// SPDX-License-Identifier: Apache-2.0
// Launch template shared by every GEMM-based kernel (plain, SiLU*mul,
// GEMM + reduce-scatter, all-gather + GEMM).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "fused/gemm_host.h"
#include "kernels/gemm_sm100.cuh"
#include "kernels/gemm_sm100_pair.cuh"

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

// ---- CTA-pair GEMM (256 x 256 tiles on two SMs) ---------------------------------
constexpr int kPairStages = 6;

// Grouping of pair-row tiles in the tile order (VCCL_GEMM_GROUP overrides
// the measured default for K): a wave of pairs then reads a compact block of
// A rows and B columns.
int pairGroupRows(int K);
// VCCL_GEMM_PAIR: 1 (default) the pair kernel where pairPreferred says so,
// 0 never, 2 for every shape of at least one pair tile.
int pairMode();
// Clusters of two that fit on the device at once with the pair kernel's
// shared memory and threads (0 if the device cannot run it).
int pairMaxClusters(const void* kernel, int smemBytes, int threads);

// True when the pair kernel finishes the shape in no more waves x tile width
// than the one-SM kernel's choice: it moves a third less data per FLOP, so
// it is taken on ties.
inline bool pairPreferred(int M, int N, int bnOverride, int pairs) {
  const int mode = pairMode();
  if (mode == 0 || bnOverride > 0 || M < kPairBM || N < kPairBN || pairs <= 0) return false;
  if (mode == 2) return true;
  const int sms = smCount();
  const int tiles2 = ((M + kPairBM - 1) / kPairBM) * ((N + kPairBN - 1) / kPairBN);
  const long cost2 = static_cast<long>((tiles2 + pairs - 1) / pairs) * kPairBN;
  const int bn = pickBN(M, N);
  const int tiles1 = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  const long cost1 = static_cast<long>((tiles1 + sms - 1) / sms) * bn;
  return cost2 <= cost1;
}

template <typename Hooks>
using PairSmemFor = PairSmem<kPairStages, 4 * Hooks::kEpiGroups>;

// Clusters of two that fit at once for this (epilogue, policy) instance.
template <typename Epi, typename Hooks = PairNoHooks>
int pairClustersFor() {
  return pairMaxClusters(reinterpret_cast<const void*>(gemmPairKernel<kPairStages, Epi, Hooks>),
                         PairSmemFor<Hooks>::kBytes, ctaThreads<Hooks>());
}

// C = A B^T on CTA pairs with epilogue `epi` and policy `hooks`.  The grid is
// `fixedPairs` clusters when > 0 (fused kernels size their counters by it;
// it must not exceed pairClustersFor), else one cluster per tile up to what
// fits.  Returns cudaErrorNotSupported if the device cannot co-schedule the
// pairs.
template <typename Epi, typename Hooks = PairNoHooks>
cudaError_t launchGemmPair(const void* A, const void* B, int M, int N, int K, const Epi& epi, cudaStream_t st,
                           int* flag = nullptr, const Hooks& hooks = Hooks{}, int fixedPairs = 0, int splits = 1) {
  using L = PairSmemFor<Hooks>;
  auto kern = gemmPairKernel<kPairStages, Epi, Hooks>;
  static std::atomic<unsigned long long> attrDone{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attrDone.load(std::memory_order_acquire) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    if (e != cudaSuccess) cudaGetLastError();
    attrDone.fetch_or(bit, std::memory_order_release);
  }
  const int maxPairs = pairMaxClusters(reinterpret_cast<const void*>(kern), L::kBytes, ctaThreads<Hooks>());
  if (maxPairs <= 0 || fixedPairs > maxPairs) return cudaErrorNotSupported;
  CUtensorMap ma, mb;
  if (!makeMapKMajor(&ma, A, M, K, kBM) || !makeMapKMajor(&mb, B, N, K, kPairBN / 2)) return cudaErrorInvalidValue;
  GemmShape s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.tilesM = (M + kPairBM - 1) / kPairBM;
  s.tilesN = (N + kPairBN - 1) / kPairBN;
  s.splits = splits < 1 ? 1 : splits;
  s.aRows = kBM;
  if (s.splits > s.numK()) return cudaErrorInvalidValue;
  const int tiles = s.tilesM * s.tilesN * s.splits;
  const int pairs = fixedPairs > 0 ? fixedPairs : tiles < maxPairs ? tiles : maxPairs;
  if (flag == nullptr) flag = errorFlag();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(ctaThreads<Hooks>()), 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, s, epi, hooks, pairGroupRows(K), flag);
}

}  // namespace gemm
}  // namespace vccl
