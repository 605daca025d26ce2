// SPDX-License-Identifier: Apache-2.0
// Host-side kernel launchers (one translation unit per kernel family so the
// template instantiations compile in parallel).
#pragma once

#include <cuda_runtime.h>

#include "kernels/coll_abi.cuh"
#include "kernels/dtypes.cuh"
#include "vccl.h"

namespace vccl {

enum class ArAlgo : int { LL = 0, TwoShot = 1, Nvls = 2, LL2 = 3, NvlsPipe = 4 };

struct LaunchCtx {
  dev::DevComm dc;
  cudaStream_t stream;
  int nblocks;     // max grid of barrier kernels
  bool nvls;
  size_t llMax;    // largest per-rank payload sent with the LL protocol
  size_t llAgMax;  // the same for all-gather (no reduction, so LL pays off further)
  int llBlocks;    // grid of every LL kernel (fixed per communicator)
  int nvlsPieces;  // pieces of a pipelined NVLS all-reduce
};

struct DeviceState;
// Launch context of a communicator's device state on stream s.
LaunchCtx launchCtxFor(const DeviceState& ds, cudaStream_t s);

inline bool aligned8(const void* a, const void* b) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 7u) == 0;
}

// redKind: dev::kSum/kProd/kMax/kMin.  Returns cudaErrorInvalidValue for an
// unsupported combination (the caller picks another algorithm).
cudaError_t launchAllReduce(const LaunchCtx& lc, ArAlgo algo, vcclDataType_t dt, int redKind,
                            const dev::CollArgs& a);
cudaError_t launchReduceScatter(const LaunchCtx& lc, vcclDataType_t dt, int redKind,
                                const dev::CollArgs& a);
cudaError_t launchAllGather(const LaunchCtx& lc, const void* send, void* recv, size_t bytes);
cudaError_t launchBroadcast(const LaunchCtx& lc, const void* send, void* recv, size_t bytes, int root,
                            bool useNvls);
cudaError_t launchP2p(const LaunchCtx& lc, const dev::P2pPlan& plan);
// Zero-copy collectives on registered windows; viaSwitch picks the NVLS
// (multimem) kernel where the buffers, datatype and operation allow it.
cudaError_t launchAllReduceWindow(const LaunchCtx& lc, vcclDataType_t dt, int redKind, const dev::WinArgs& w,
                                  bool viaSwitch);
cudaError_t launchAllGatherWindow(const LaunchCtx& lc, const dev::WinArgs& w);
cudaError_t launchAllToAllvWindow(const LaunchCtx& lc, const dev::WinArgs& w, const dev::A2aTable& t, int esz);
cudaError_t launchBroadcastWindow(const LaunchCtx& lc, const dev::WinArgs& w, int root);
cudaError_t launchReduceScatterWindow(const LaunchCtx& lc, vcclDataType_t dt, int redKind, const dev::WinArgs& w,
                                      bool viaSwitch);
// Single-rank helpers: dst = src * scale (float types) or plain copy.
cudaError_t launchScaleCopy(cudaStream_t s, vcclDataType_t dt, void* dst, const void* src, size_t count,
                            double scale);

bool nvlsSupports(vcclDataType_t dt, int redKind);
// Pipelined NVLS all-reduce geometry: bytes per staging slot, and the per-rank
// chunk of one piece (a multiple of 16, n * chunk fits in a slot).
size_t nvlsPipeSlotBytes(size_t dataBytes);
size_t nvlsPipeChunk(size_t bytes, int n, int pieces, size_t dataBytes);
int gridFor(size_t bytes, int maxBlocks);

}  // namespace vccl
