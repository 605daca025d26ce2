// SPDX-License-Identifier: Apache-2.0
// Zero-copy collectives on registered windows.
//
// A window is user memory (from vcclMemAlloc) that every rank of the
// communicator has mapped, and, when the node supports NVLS, bound to a
// multicast object (vcclCommWindowRegister).  When a collective's buffers
// lie in windows, the kernels below read the peers' send buffers and write
// the peers' receive buffers in place: there is no staging copy in or out,
// which the staging algorithms pay on every byte.  The reference registers
// buffers only to pin them for its transport (reference:
// src/core/comm.cc:180-244); mapping them into every peer is what makes the
// in-place access possible here.
//
// Usage rule (checked): every rank passes buffers at the same offsets of
// its windows and the same count.  Each block publishes its call's
// descriptor before the start barrier and compares the peers' after it; a
// mismatch is recorded as an error and every rank returns without touching
// data.  The barrier at the end keeps a rank from returning (and, say,
// overwriting its send buffer) while a peer still reads it.
#pragma once

#include "kernels/collectives.cuh"

namespace vccl {
namespace dev {

// Publish block blk's descriptor, meet the peers, compare.  Fills
// scalars[q] with rank q's PreMulSum factor.  False: the block must return
// (barrier failure, or a mismatch that every rank sees as well).
__device__ __forceinline__ bool winStart(const DevComm& c, int blk, const WinArgs& w, double* scalars) {
  __shared__ int sBad;
  if (threadIdx.x == 0) {
    WinDesc* d = ctrlAt<WinDesc>(c, c.rank, kWinDescOff) + blk;
    d->sendOff = w.sendOff;
    d->recvOff = w.recvOff;
    d->count = w.count;
    d->scalar = w.premul ? w.scalar : 1.0;
    sBad = 0;
  }
  // The barrier's release store covers the descriptor written above.
  if (!blockBarrier(c, blk, kWhereStart)) return false;
  const int t = threadIdx.x;
  if (t < c.nranks) {
    const volatile WinDesc* d = ctrlAt<WinDesc>(c, t, kWinDescOff) + blk;
    if (d->sendOff != w.sendOff || d->recvOff != w.recvOff || d->count != w.count) sBad = 1;
    scalars[t] = d->scalar;
  }
  __syncthreads();
  if (sBad) {
    if (threadIdx.x == 0) recordFailure(c, kErrBadArg, kWhereWindow, static_cast<uint32_t>(blk));
    return false;
  }
  return true;
}

// Sum of every rank's element i (each scaled by its factor), read at
// send[q] + srcOff, for elements [lo, hi), stored to every rank's recv (or
// to this rank's only).  Only this rank reduces these elements; it folds
// the sources starting with its own.
template <typename T, int K, bool VEC>
__device__ __forceinline__ void winReduceBroadcast(const WinArgs& w, size_t srcOff, int n, int me, size_t lo,
                                                   size_t hi, const double* scalars, bool out0Only) {
  constexpr int U = sizeof(T) == 1 ? 2 : 4;  // 16 fp32 accumulators per pack of 8-bit types
  using E = Elem<T>;
  const size_t nthr = blockDim.x;
  const int outs = out0Only ? 1 : n;
  size_t done = lo;
  if constexpr (VEC) {
    constexpr size_t PK = 16 / sizeof(T);
    const size_t p0 = lo / PK, p1 = hi / PK;  // lo is a multiple of PK
    size_t i = p0 + threadIdx.x;
    for (; i < p1; i += U * nthr) {
      Pack<T> acc[U];
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; u++)
        if (i + u * nthr < p1) raw[u] = ldCG(w.send[me] + srcOff + (i + u * nthr) * 16);
#pragma unroll
      for (int u = 0; u < U; u++) {
        acc[u].load(raw[u]);
        if (w.premul) acc[u].scale(scalars[me]);
      }
#pragma unroll 1
      for (int k = 1; k < n; k++) {
        int q = me + k;
        if (q >= n) q -= n;
#pragma unroll
        for (int u = 0; u < U; u++)
          if (i + u * nthr < p1) raw[u] = ldCG(w.send[q] + srcOff + (i + u * nthr) * 16);
#pragma unroll
        for (int u = 0; u < U; u++) acc[u].template fold<K>(scaledRaw<T>(raw[u], w.premul != 0, scalars[q]));
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        if (i + u * nthr >= p1) break;
        if (w.avg) acc[u].scale(1.0 / n);
        const uint4 r = acc[u].pack();
        for (int k = 0; k < outs; k++) {
          int q = me + k;
          if (q >= n) q -= n;
          stG(w.recv[q] + (i + u * nthr) * 16, r);
        }
      }
    }
    done = p1 * PK > lo ? p1 * PK : lo;
  }
  for (size_t i = done + threadIdx.x; i < hi; i += nthr) {
    typename E::Acc acc = E::toAcc(reinterpret_cast<const T*>(w.send[me] + srcOff)[i]);
    if (w.premul) acc = scaleAcc<T>(acc, scalars[me]);
    for (int k = 1; k < n; k++) {
      int q = me + k;
      if (q >= n) q -= n;
      typename E::Acc v = E::toAcc(reinterpret_cast<const T*>(w.send[q] + srcOff)[i]);
      if (w.premul) v = E::toAcc(E::fromAcc(scaleAcc<T>(v, scalars[q])));
      acc = combine<T, K>(acc, v);
    }
    if (w.avg) acc = scaleAcc<T>(acc, 1.0 / n);
    const T r = E::fromAcc(acc);
    for (int k = 0; k < outs; k++) {
      int q = me + k;
      if (q >= n) q -= n;
      reinterpret_cast<T*>(w.recv[q])[i] = r;
    }
  }
}

// All-reduce, both buffers in windows: rank r reduces chunk r straight from
// the peers' send buffers and writes the result into every rank's receive
// buffer.  Per rank (n-1)/n of the message crosses NVLink each way.
template <typename T, int K, bool VEC>
__global__ void __launch_bounds__(512) allReduceWin(DevComm c, WinArgs w) {
  __shared__ double sScale[kMaxRanks];
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (!winStart(c, blk, w, sScale)) return;
  constexpr size_t PK = VEC ? 16 / sizeof(T) : 1;
  const size_t ce = rankChunk(w.count, n, PK);
  size_t s0, s1;
  blockRange(ce, G, blk, PK, &s0, &s1);
  const size_t lo = me * ce + s0;
  const size_t hiRaw = me * ce + s1;
  const size_t hi = hiRaw < w.count ? hiRaw : w.count;
  if (lo < hi) winReduceBroadcast<T, K, VEC>(w, 0, n, me, lo, hi, sScale, false);
  (void)blockBarrier(c, blk, kWhereWindow);
}

// All-reduce through the switch: multimem.ld_reduce of chunk r from the
// send buffers' multicast address, multimem.st to the receive buffers'
// (the switch reduces and fans out; nothing is staged).  Bytes, offsets
// and both multicast addresses are multiples of 16.
template <typename T, int K>
__global__ void __launch_bounds__(512) allReduceWinNvls(DevComm c, WinArgs w) {
  __shared__ double sScale[kMaxRanks];
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (!winStart(c, blk, w, sScale)) return;
  if constexpr (HasMultimem<T, K>::value) {
    const size_t total = w.count * sizeof(T);
    const size_t cb = rankChunk(total, n, 16);
    size_t s0, s1;
    blockRange(cb, G, blk, 16, &s0, &s1);
    const size_t lo = me * cb + s0;
    const size_t hiRaw = me * cb + s1;
    const size_t hi = hiRaw < total ? hiRaw : total;
    if (lo < hi) nvlsReduceRange<T, K, 8>(w.mcSend, w.mcRecv, lo, hi, w.avg != 0, n, threadIdx.x, blockDim.x);
  }
  fenceProxyAlias();
  (void)blockBarrier(c, blk, kWhereWindow);
}

// All-gather, receive buffer in a window: every rank writes its block into
// every rank's receive buffer at offset rank * bytes, with one multimem.st
// per 16 bytes when the receive buffers are multicast-bound (one copy
// leaves the GPU, the switch fans it out), else with a store per peer.
// w.send[me] is the local send buffer (it need not be in a window).
__global__ void __launch_bounds__(512) allGatherWin(DevComm c, WinArgs w) {
  __shared__ double sScale[kMaxRanks];
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (!winStart(c, blk, w, sScale)) return;
  const size_t bytes = w.count;
  size_t lo, hi;
  blockRange(bytes, G, blk, 16, &lo, &hi);
  if (lo < hi) {
    const char* src = w.send[me] + lo;
    if (w.mcRecv != nullptr) {
      // bytes, the send buffer and the receive offset are multiples of 16 here
      char* dst = w.mcRecv + me * bytes + lo;
      const size_t units = (hi - lo) / 16;
      const size_t nthr = blockDim.x;
      size_t i = threadIdx.x;
      for (; i + (kUnroll - 1) * nthr < units; i += kUnroll * nthr) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) v[u] = ldCG(src + (i + u * nthr) * 16);
#pragma unroll
        for (int u = 0; u < kUnroll; u++) multimemStore16(dst + (i + u * nthr) * 16, v[u]);
      }
      for (; i < units; i += nthr) multimemStore16(dst + i * 16, ldCG(src + i * 16));
    } else {
      for (int k = 0; k < n; k++) {
        int q = me + k;
        if (q >= n) q -= n;
        copyAny(w.recv[q] + me * bytes + lo, src, hi - lo);
      }
    }
  }
  fenceProxyAlias();
  (void)blockBarrier(c, blk, kWhereWindow);
}

// Broadcast, receive buffer in a window: the root writes its buffer into
// every rank's receive buffer, with one multimem.st per 16 bytes when the
// receive buffers are multicast-bound (one copy leaves the root), else with a
// store per rank.  The other ranks only take part in the barriers.
__global__ void __launch_bounds__(512) broadcastWin(DevComm c, WinArgs w, int root) {
  __shared__ double sScale[kMaxRanks];
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (!winStart(c, blk, w, sScale)) return;
  const size_t bytes = w.count;
  size_t lo, hi;
  blockRange(bytes, G, blk, 16, &lo, &hi);
  if (me == root && lo < hi) {
    const char* src = w.send[me] + lo;
    if (w.mcRecv != nullptr) {
      // bytes, the send buffer and the receive offset are multiples of 16 here
      char* dst = w.mcRecv + lo;
      for (size_t i = threadIdx.x; i < (hi - lo) / 16; i += blockDim.x)
        multimemStore16(dst + i * 16, ldCG(src + i * 16));
    } else {
      for (int k = 0; k < n; k++) {
        int q = me + k;
        if (q >= n) q -= n;
        copyAny(w.recv[q] + lo, src, hi - lo);
      }
    }
  }
  fenceProxyAlias();
  (void)blockBarrier(c, blk, kWhereWindow);
}

// All-to-all(v), receive buffer in a window: every rank publishes where it
// wants each source's block (its receive count and displacement for that
// source) before the start barrier; every sender reads its entry at each
// destination, checks that its send count matches, and writes its block
// straight into the destination's receive buffer.  w.recv[q] is rank q's
// receive buffer, w.send[me] the local send buffer; counts are in elements
// of esz bytes.  A count mismatch is recorded as an error; the ranks that
// saw none still meet at the end barrier, whose waits then run out.
__global__ void __launch_bounds__(512) allToAllvWin(DevComm c, WinArgs w, A2aTable t, int esz) {
  __shared__ double sScale[kMaxRanks];
  __shared__ uint64_t sDispl[kMaxRanks];
  __shared__ int sBad;
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (threadIdx.x < n) {
    uint64_t* e = ctrlAt<uint64_t>(c, me, kWinA2aOff) + (static_cast<size_t>(blk) * kMaxRanks + threadIdx.x) * 2;
    e[0] = t.rc[threadIdx.x];
    e[1] = t.rd[threadIdx.x];
  }
  if (threadIdx.x == 0) sBad = 0;
  // winStart's barrier begins with a block-wide sync and releases the table too.
  if (!winStart(c, blk, w, sScale)) return;
  if (threadIdx.x < n) {
    const volatile uint64_t* e =
        ctrlAt<uint64_t>(c, threadIdx.x, kWinA2aOff) + (static_cast<size_t>(blk) * kMaxRanks + me) * 2;
    if (e[0] != t.sc[threadIdx.x]) sBad = 1;
    sDispl[threadIdx.x] = e[1];
  }
  __syncthreads();
  if (sBad) {
    if (threadIdx.x == 0) recordFailure(c, kErrBadArg, kWhereWindow, static_cast<uint32_t>(blk));
    return;
  }
  for (int k = 0; k < n; k++) {
    int q = me + k;
    if (q >= n) q -= n;
    const size_t bytes = t.sc[q] * esz;
    size_t lo, hi;
    blockRange(bytes, G, blk, 16, &lo, &hi);
    if (lo < hi) copyAny(w.recv[q] + sDispl[q] * esz + lo, w.send[me] + t.sd[q] * esz + lo, hi - lo);
  }
  (void)blockBarrier(c, blk, kWhereWindow);
}

// Reduce-scatter, send buffer in a window: rank r reduces its chunk
// (elements [r*count, (r+1)*count) of every send buffer) straight from the
// peers, through the switch when the send buffers are multicast-bound (and
// no PreMulSum), into its own receive buffer (which need not be in a window).
template <typename T, int K, bool VEC>
__global__ void __launch_bounds__(512) reduceScatterWin(DevComm c, WinArgs w, int useNvls) {
  __shared__ double sScale[kMaxRanks];
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (!winStart(c, blk, w, sScale)) return;
  constexpr size_t PK = VEC ? 16 / sizeof(T) : 1;
  const size_t rc = w.count;
  const size_t esz = sizeof(T);
  size_t s0, s1;
  blockRange(rc, G, blk, PK, &s0, &s1);
  bool viaSwitch = false;
  if constexpr (HasMultimem<T, K>::value) viaSwitch = useNvls != 0;
  if (s0 < s1 && viaSwitch) {
    if constexpr (HasMultimem<T, K>::value) {
      // rc * sizeof(T), the offsets and the buffers are multiples of 16 here.
      const char* src = w.mcSend + me * rc * esz;
      char* dst = w.recv[me];
      const size_t u0 = s0 * esz / 16, u1 = (s1 * esz + 15) / 16;
      for (size_t i = u0 + threadIdx.x; i < u1; i += blockDim.x) {
        uint4 v = Multimem<T, K>::ldReduce(src + i * 16);
        if (w.avg) {
          Pack<T> p;
          p.load(v);
          p.scale(1.0 / n);
          v = p.pack();
        }
        stG(dst + i * 16, v);
      }
    }
  } else if (s0 < s1) {
    // Point to point: sources read at this rank's chunk, element indices
    // relative to the chunk, one output (this rank's buffer).
    winReduceBroadcast<T, K, VEC>(w, me * rc * esz, n, me, s0, s1, sScale, true);
  }
  fenceProxyAlias();
  (void)blockBarrier(c, blk, kWhereWindow);
}

}  // namespace dev
}  // namespace vccl
