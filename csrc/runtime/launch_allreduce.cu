// SPDX-License-Identifier: Apache-2.0
// All-reduce / reduce launchers (LL, two-hop LL, two-shot, NVLS); the
// algorithm is chosen in collectives.cc, as the reference's dispatcher
// chooses ring or recursive doubling (reference:
// src/core/collectives.cc:505-555, reduce chain :557-620).
#include "kernels/collectives.cuh"
#include "runtime/dispatch.cuh"
#include "runtime/launch.h"

namespace vccl {

constexpr int kThreads = 512;

int gridFor(size_t bytes, int maxBlocks) {
  // ~32 KiB per block: each block keeps 8 x 16 B loads per thread in flight
  // (64 KiB at 512 threads), so this fills the NVLink pipe with enough
  // blocks while small messages do not pay for idle ones.
  size_t g = (bytes + (32u << 10) - 1) / (32u << 10);
  if (g < 1) g = 1;
  if (g > static_cast<size_t>(maxBlocks)) g = maxBlocks;
  return static_cast<int>(g);
}

size_t nvlsPipeSlotBytes(size_t dataBytes) {
  return (dataBytes - 16 * dev::kMaxRanks) / dev::kPipeSlots / 16 * 16;
}

size_t nvlsPipeChunk(size_t bytes, int n, int pieces, size_t dataBytes) {
  const size_t maxCb = nvlsPipeSlotBytes(dataBytes) / n / 16 * 16;
  const size_t piece = (bytes + pieces - 1) / pieces;
  size_t cb = ((piece + n - 1) / n + 15) / 16 * 16;
  if (cb > maxCb) cb = maxCb;
  return cb < 16 ? 16 : cb;
}

bool nvlsSupports(vcclDataType_t dt, int k) {
  if (k == dev::kSum) return dt == vcclFloat32 || dt == vcclBfloat16 || dt == vcclFloat16;
  if (k == dev::kMin || k == dev::kMax) return dt == vcclBfloat16 || dt == vcclFloat16;
  return false;
}

cudaError_t launchAllReduce(const LaunchCtx& lc, ArAlgo algo, vcclDataType_t dt, int redKind,
                            const dev::CollArgs& a) {
  const size_t esz = vcclTypeSize(dt);
  const size_t bytes = a.count * esz;
  const int n = lc.dc.nranks;
  if (algo == ArAlgo::LL) {
    if (bytes > dev::kLLMaxBytes ||
        ((reinterpret_cast<uintptr_t>(a.send) | reinterpret_cast<uintptr_t>(a.recv)) & 7u) != 0 || a.root >= 0)
      return cudaErrorInvalidValue;
    VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
      dev::allReduceLL<T, K><<<lc.llBlocks, kThreads, 0, lc.stream>>>(lc.dc, a);
    }))
    return cudaGetLastError();
  }
  if (algo == ArAlgo::LL2) {
    const size_t words = (bytes + 7) / 8;
    if ((words + n - 1) / n * 8 > dev::kLLMaxBytes ||
        ((reinterpret_cast<uintptr_t>(a.send) | reinterpret_cast<uintptr_t>(a.recv)) & 7u) != 0 || a.root >= 0)
      return cudaErrorInvalidValue;
    VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
      dev::allReduceLL2<T, K><<<lc.llBlocks, kThreads, 0, lc.stream>>>(lc.dc, a);
    }))
    return cudaGetLastError();
  }
  if (algo == ArAlgo::Nvls) {
    if (!lc.nvls || !nvlsSupports(dt, redKind) || a.root >= 0) return cudaErrorInvalidValue;
    const size_t roundBytes = (lc.dc.dataBytes - 16 * dev::kMaxRanks) / 16 * 16;
    const int g = gridFor(bytes / n, lc.nblocks);
    VCCL_DISPATCH_MULTIMEM(dt, redKind, {
      dev::allReduceNvls<T, K><<<g, kThreads, 0, lc.stream>>>(lc.dc, a, roundBytes);
    })
    return cudaGetLastError();
  }
  if (algo == ArAlgo::NvlsPipe) {
    if (!lc.nvls || !nvlsSupports(dt, redKind) || a.root >= 0) return cudaErrorInvalidValue;
    const size_t cb = nvlsPipeChunk(bytes, n, lc.nvlsPieces, lc.dc.dataBytes);
    const size_t slotBytes = nvlsPipeSlotBytes(lc.dc.dataBytes);
    const int g = gridFor(bytes / n, lc.nblocks);
    VCCL_DISPATCH_MULTIMEM(dt, redKind, {
      dev::allReduceNvlsPipe<T, K><<<g, dev::kPipeThreads, 0, lc.stream>>>(lc.dc, a, cb, slotBytes);
    })
    return cudaGetLastError();
  }
  // Two-shot (all-reduce, or reduce when a.root >= 0).
  const bool vec = ((reinterpret_cast<uintptr_t>(a.send) | reinterpret_cast<uintptr_t>(a.recv)) & 15u) == 0;
  const size_t pk = 16 / esz;
  size_t slotElems = lc.dc.dataBytes / (n + 1) / esz;
  slotElems = slotElems / pk * pk;
  const int g = gridFor(bytes / n, lc.nblocks);
  VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
    if (vec)
      dev::allReduceTwoShot<T, K, true><<<g, kThreads, 0, lc.stream>>>(lc.dc, a, slotElems);
    else
      dev::allReduceTwoShot<T, K, false><<<g, kThreads, 0, lc.stream>>>(lc.dc, a, slotElems);
  }))
  return cudaGetLastError();
}

}  // namespace vccl
