// SPDX-License-Identifier: Apache-2.0
// Reduce-scatter, all-gather, broadcast, point-to-point and single-rank
// launchers (reference counterparts: src/core/collectives.cc:283-349
// reduce-scatter, :243-281 all-gather dispatcher, :622-649 broadcast chain,
// :651-740 gather / scatter / all-to-all, :886-905 send / recv).
#include "kernels/movement.cuh"
#include "runtime/dispatch.cuh"
#include "runtime/launch.h"

namespace vccl {

namespace {
constexpr int kThreads = 512;

template <typename T>
__global__ void scaleCopyKernel(T* dst, const T* src, size_t n, double s) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = dev::scaledElem<T>(src[i], true, s);
}
}  // namespace

cudaError_t launchReduceScatter(const LaunchCtx& lc, vcclDataType_t dt, int redKind, const dev::CollArgs& a) {
  const size_t esz = vcclTypeSize(dt);
  const int n = lc.dc.nranks;
  const size_t chunkBytes = a.count * esz;
  if (chunkBytes <= lc.llMax && chunkBytes % 8 == 0 && aligned8(a.send, a.recv)) {
    VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
      dev::reduceScatterLL<T, K><<<lc.llBlocks, kThreads, 0, lc.stream>>>(lc.dc, a);
    }))
    return cudaGetLastError();
  }
  const bool vec = ((reinterpret_cast<uintptr_t>(a.send) | reinterpret_cast<uintptr_t>(a.recv)) & 15u) == 0 &&
                   (a.count * esz) % 16 == 0;
  const size_t pk = 16 / esz;
  size_t slotElems = (lc.dc.dataBytes / 2) / n / esz;
  slotElems = slotElems / pk * pk;
  const int g = gridFor(a.count * esz, lc.nblocks);
  VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
    if (vec)
      dev::reduceScatterPush<T, K, true><<<g, kThreads, 0, lc.stream>>>(lc.dc, a, slotElems);
    else
      dev::reduceScatterPush<T, K, false><<<g, kThreads, 0, lc.stream>>>(lc.dc, a, slotElems);
  }))
  return cudaGetLastError();
}

cudaError_t launchAllGather(const LaunchCtx& lc, const void* send, void* recv, size_t bytes) {
  if (bytes <= lc.llAgMax && bytes % 8 == 0 && aligned8(send, recv)) {
    dev::allGatherLL<<<lc.llBlocks, kThreads, 0, lc.stream>>>(lc.dc, static_cast<const char*>(send),
                                                                  static_cast<char*>(recv), bytes);
    return cudaGetLastError();
  }
  const int g = gridFor(bytes, lc.nblocks);
  dev::allGatherPull<<<g, kThreads, 0, lc.stream>>>(lc.dc, static_cast<const char*>(send),
                                                    static_cast<char*>(recv), bytes);
  return cudaGetLastError();
}

cudaError_t launchBroadcast(const LaunchCtx& lc, const void* send, void* recv, size_t bytes, int root,
                            bool useNvls) {
  if (bytes <= lc.llMax && bytes % 8 == 0 && aligned8(send, recv)) {
    dev::broadcastLL<<<lc.llBlocks, kThreads, 0, lc.stream>>>(lc.dc, static_cast<const char*>(send),
                                                                  static_cast<char*>(recv), bytes, root);
    return cudaGetLastError();
  }
  const int g = gridFor(bytes, lc.nblocks);
  if (useNvls && lc.nvls)
    dev::broadcastNvls<<<g, kThreads, 0, lc.stream>>>(lc.dc, static_cast<const char*>(send),
                                                      static_cast<char*>(recv), bytes, root);
  else
    dev::broadcastPull<<<g, kThreads, 0, lc.stream>>>(lc.dc, static_cast<const char*>(send),
                                                      static_cast<char*>(recv), bytes, root);
  return cudaGetLastError();
}

cudaError_t launchP2p(const LaunchCtx& lc, const dev::P2pPlan& plan) {
  if (plan.nwork == 0) return cudaSuccess;
  dev::p2pKernel<<<plan.nwork, kThreads, 0, lc.stream>>>(lc.dc, plan);
  return cudaGetLastError();
}

cudaError_t launchScaleCopy(cudaStream_t s, vcclDataType_t dt, void* dst, const void* src, size_t count,
                            double scale) {
  if (count == 0) return cudaSuccess;
  const size_t esz = vcclTypeSize(dt);
  if (scale == 1.0 || !(dt == vcclFloat16 || dt == vcclFloat32 || dt == vcclFloat64 || dt == vcclBfloat16 ||
                        dt == vcclFloat8e4m3 || dt == vcclFloat8e5m2)) {
    if (dst == src) return cudaSuccess;
    return cudaMemcpyAsync(dst, src, count * esz, cudaMemcpyDefault, s);
  }
  size_t blocks = (count + kThreads - 1) / kThreads;
  if (blocks > 1024) blocks = 1024;
  VCCL_DISPATCH_TYPE(dt, {
    scaleCopyKernel<T><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(static_cast<T*>(dst),
                                                                         static_cast<const T*>(src), count,
                                                                         scale);
  })
  return cudaGetLastError();
}

}  // namespace vccl
