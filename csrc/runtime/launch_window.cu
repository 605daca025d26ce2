// SPDX-License-Identifier: Apache-2.0
// Launchers of the zero-copy window collectives (csrc/kernels/window.cuh).
// The reference has no counterpart: its registered buffers are pinned host
// memory for the transport (reference: src/core/comm.cc:180-244).
#include "kernels/window.cuh"
#include "runtime/dispatch.cuh"
#include "runtime/launch.h"

namespace vccl {

namespace {
constexpr int kThreads = 512;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

cudaError_t launchAllReduceWindow(const LaunchCtx& lc, vcclDataType_t dt, int redKind, const dev::WinArgs& w,
                                  bool viaSwitch) {
  const size_t esz = vcclTypeSize(dt);
  const int n = lc.dc.nranks;
  const size_t bytes = w.count * esz;
  const int g = gridFor(bytes / n, lc.nblocks);
  if (viaSwitch) {
    if (w.mcSend == nullptr || w.mcRecv == nullptr || w.premul || !nvlsSupports(dt, redKind) || bytes % 16 != 0 ||
        !aligned16(w.mcSend) || !aligned16(w.mcRecv))
      return cudaErrorInvalidValue;
    VCCL_DISPATCH_MULTIMEM(dt, redKind, { dev::allReduceWinNvls<T, K><<<g, kThreads, 0, lc.stream>>>(lc.dc, w); })
    return cudaGetLastError();
  }
  // Vector path when every rank's buffers sit on 16-byte boundaries (the
  // offsets agree across ranks, and the windows start on allocation
  // granules, so checking this rank's pointers is enough).
  bool vec = true;
  for (int q = 0; q < n; q++) vec = vec && aligned16(w.send[q]) && aligned16(w.recv[q]);
  VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
    if (vec)
      dev::allReduceWin<T, K, true><<<g, kThreads, 0, lc.stream>>>(lc.dc, w);
    else
      dev::allReduceWin<T, K, false><<<g, kThreads, 0, lc.stream>>>(lc.dc, w);
  }))
  return cudaGetLastError();
}

cudaError_t launchAllGatherWindow(const LaunchCtx& lc, const dev::WinArgs& w) {
  const int g = gridFor(w.count, lc.nblocks);
  dev::WinArgs v = w;
  // One multimem store per 16 bytes needs 16-byte units on both sides.
  if (v.mcRecv != nullptr && (w.count % 16 != 0 || !aligned16(w.send[lc.dc.rank]) || !aligned16(w.mcRecv)))
    v.mcRecv = nullptr;
  dev::allGatherWin<<<g, kThreads, 0, lc.stream>>>(lc.dc, v);
  return cudaGetLastError();
}

cudaError_t launchBroadcastWindow(const LaunchCtx& lc, const dev::WinArgs& w, int root) {
  const int g = gridFor(w.count, lc.nblocks);
  dev::WinArgs v = w;
  if (v.mcRecv != nullptr && (w.count % 16 != 0 || !aligned16(w.send[lc.dc.rank]) || !aligned16(w.mcRecv)))
    v.mcRecv = nullptr;
  // Every rank must pick the same kernel shape; only the root reads mcRecv,
  // so the choice above matters on the root alone.
  dev::broadcastWin<<<g, kThreads, 0, lc.stream>>>(lc.dc, v, root);
  return cudaGetLastError();
}

cudaError_t launchAllToAllvWindow(const LaunchCtx& lc, const dev::WinArgs& w, const dev::A2aTable& t, int esz) {
  // Block counts differ between ranks, so the grid cannot follow them: every
  // rank launches the full barrier grid (block b meets block b of the peers).
  dev::allToAllvWin<<<lc.nblocks, kThreads, 0, lc.stream>>>(lc.dc, w, t, esz);
  return cudaGetLastError();
}

cudaError_t launchReduceScatterWindow(const LaunchCtx& lc, vcclDataType_t dt, int redKind, const dev::WinArgs& w,
                                      bool viaSwitch) {
  const size_t esz = vcclTypeSize(dt);
  const int n = lc.dc.nranks;
  const int me = lc.dc.rank;
  const size_t chunk = w.count * esz;
  const int g = gridFor(chunk, lc.nblocks);
  bool vec = chunk % 16 == 0 && aligned16(w.recv[me]);
  for (int q = 0; q < n; q++) vec = vec && aligned16(w.send[q]);
  const int nv = viaSwitch && vec && w.mcSend != nullptr && aligned16(w.mcSend) && !w.premul &&
                 nvlsSupports(dt, redKind);
  VCCL_DISPATCH_TYPE(dt, VCCL_DISPATCH_OP(redKind, {
    if (vec)
      dev::reduceScatterWin<T, K, true><<<g, kThreads, 0, lc.stream>>>(lc.dc, w, nv);
    else
      dev::reduceScatterWin<T, K, false><<<g, kThreads, 0, lc.stream>>>(lc.dc, w, 0);
  }))
  return cudaGetLastError();
}

}  // namespace vccl
