// SPDX-License-Identifier: Apache-2.0
// Data-movement kernels without reduction: all-gather, broadcast and the
// point-to-point rings (non-template kernels; included by one translation
// unit only).
//
// Replaces the reference's ring / recursive-doubling / Bruck all-gather,
// chain broadcast and pairwise point-to-point exchanges (reference:
// src/core/collectives.cc:127-281, :622-740) with pull-based copies over
// NVLink and flow-controlled slot rings.
#pragma once

#include "kernels/collectives.cuh"

namespace vccl {
namespace dev {

// ---------------------------------------------------------------------------
// All-gather: each rank stages its block, peers pull.  Halves alternate.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) allGatherPull(DevComm c, const char* send, char* recv, size_t bytes) {
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  if (!blockBarrier(c, blk, kWhereStart)) return;
  const size_t half = (c.dataBytes / 2) / 16 * 16;
  char* ownOut = recv + me * bytes;
  int k = 0;
  for (size_t off = 0; off < bytes; off += half, k++) {
    const size_t m = (bytes - off) < half ? (bytes - off) : half;
    size_t lo, hi;
    roundRange(bytes < half ? bytes : half, m, G, blk, 16, &lo, &hi);
    const size_t hoff = (k & 1) * half;
    if (lo < hi) {
      copyAny(c.data[me] + hoff + lo, send + off + lo, hi - lo);
      if (ownOut != send) copyAny(ownOut + off + lo, send + off + lo, hi - lo);
    }
    if (!blockBarrier(c, blk, kWhereGather)) return;
    if (lo < hi) {
      for (int s = 1; s < n; s++) {
        const int q = (me + s) % n;
        copyAny(recv + q * bytes + off + lo, c.data[q] + hoff + lo, hi - lo);
      }
    }
  }
}

// LL all-gather: every rank stores its block as LL lines into every peer's
// slot; one NVLink hop, no barrier.  bytes % 8 == 0, 8-byte aligned buffers,
// bytes <= kLLMaxBytes.
__global__ void __launch_bounds__(512) allGatherLL(DevComm c, const char* send, char* recv, size_t bytes) {
  const uint32_t e = llEpoch(c);
  const uint32_t par = e & 1u;
  const int n = c.nranks, me = c.rank;
  const size_t words = bytes / 8;
  size_t w0, w1;
  blockRange(words, gridDim.x, blockIdx.x, 1, &w0, &w1);
  char* own = recv + me * bytes;
  constexpr int U = kLLUnroll;
  const size_t nthr = blockDim.x;
  for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
    uint64_t word[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      if (b + u * nthr < w1) word[u] = *reinterpret_cast<const uint64_t*>(send + (b + u * nthr) * 8);
    for (int k = 1; k < n; k++) {
      char* dst = llSlot(c, (me + k) % n, par, me);
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) stVolatile16(dst + (b + u * nthr) * 16, llLine(word[u], e));
    }
    if (own != send) {
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) *reinterpret_cast<uint64_t*>(own + (b + u * nthr) * 8) = word[u];
    }
  }
  for (int k = 1; k < n; k++) {
    const int p = (me + k) % n;
    const char* src = llSlot(c, me, par, p);
    for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
      uint64_t v[U];
      if (!llWaitU<U>(c, src, b, nthr, w1, e, v)) return;
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) *reinterpret_cast<uint64_t*>(recv + p * bytes + (b + u * nthr) * 8) = v[u];
    }
  }
}

// LL broadcast: the root stores LL lines into every peer's slot.  Reusing
// an LL slot two calls later is safe only if, in every LL call, each rank
// hears from every other rank (then finishing call k+1 proves every peer
// finished call k).  Broadcast data only flows from the root, so every
// rank also exchanges a one-line token with every peer, in the second-hop
// LL region that broadcast does not otherwise use.
__global__ void __launch_bounds__(512) broadcastLL(DevComm c, const char* send, char* recv, size_t bytes, int root) {
  const uint32_t e = llEpoch(c);
  const uint32_t par = e & 1u;
  const int n = c.nranks, me = c.rank;
  const size_t words = bytes / 8;
  size_t w0, w1;
  blockRange(words, gridDim.x, blockIdx.x, 1, &w0, &w1);
  const int p = threadIdx.x;
  if (p < n && p != me) {
    const uint4 token = make_uint4(0, e, 0, e);
    stVolatile16(llResSlot(c, p, par, me) + blockIdx.x * 16, token);
  }
  constexpr int U = kLLUnroll;
  const size_t nthr = blockDim.x;
  if (me == root) {
    for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
      uint64_t word[U];
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) word[u] = *reinterpret_cast<const uint64_t*>(send + (b + u * nthr) * 8);
      for (int k = 1; k < n; k++) {
        char* dst = llSlot(c, (me + k) % n, par, me);
#pragma unroll
        for (int u = 0; u < U; u++)
          if (b + u * nthr < w1) stVolatile16(dst + (b + u * nthr) * 16, llLine(word[u], e));
      }
      if (recv != send) {
#pragma unroll
        for (int u = 0; u < U; u++)
          if (b + u * nthr < w1) *reinterpret_cast<uint64_t*>(recv + (b + u * nthr) * 8) = word[u];
      }
    }
  } else {
    const char* src = llSlot(c, me, par, root);
    for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
      uint64_t v[U];
      if (!llWaitU<U>(c, src, b, nthr, w1, e, v)) return;
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) *reinterpret_cast<uint64_t*>(recv + (b + u * nthr) * 8) = v[u];
    }
  }
  if (p < n && p != me) {
    uint64_t token;
    llWait(c, llResSlot(c, me, par, p) + blockIdx.x * 16, e, &token);
  }
}

// ---------------------------------------------------------------------------
// Broadcast.  Pull: root stages, everyone pulls.  NVLS: root stores once
// through the multicast address, every rank copies out locally.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) broadcastPull(DevComm c, const char* send, char* recv, size_t bytes,
                                                     int root) {
  const int blk = blockIdx.x, G = gridDim.x, me = c.rank;
  if (!blockBarrier(c, blk, kWhereStart)) return;
  const size_t half = (c.dataBytes / 2) / 16 * 16;
  int k = 0;
  for (size_t off = 0; off < bytes; off += half, k++) {
    const size_t m = (bytes - off) < half ? (bytes - off) : half;
    size_t lo, hi;
    roundRange(bytes < half ? bytes : half, m, G, blk, 16, &lo, &hi);
    const size_t hoff = (k & 1) * half;
    if (me == root && lo < hi) {
      copyAny(c.data[root] + hoff + lo, send + off + lo, hi - lo);
      if (recv != send) copyAny(recv + off + lo, send + off + lo, hi - lo);
    }
    if (!blockBarrier(c, blk, kWhereGather)) return;
    if (me != root && lo < hi) copyAny(recv + off + lo, c.data[root] + hoff + lo, hi - lo);
  }
}

__global__ void __launch_bounds__(512) broadcastNvls(DevComm c, const char* send, char* recv, size_t bytes,
                                                     int root) {
  const int blk = blockIdx.x, G = gridDim.x, me = c.rank;
  if (!blockBarrier(c, blk, kWhereStart)) return;
  const size_t half = (c.dataBytes / 2) / 16 * 16;
  int k = 0;
  for (size_t off = 0; off < bytes; off += half, k++) {
    const size_t m = (bytes - off) < half ? (bytes - off) : half;
    size_t lo, hi;
    roundRange(bytes < half ? bytes : half, m, G, blk, 16, &lo, &hi);
    const size_t hoff = (k & 1) * half;
    if (me == root && lo < hi) {
      const bool al = (reinterpret_cast<uintptr_t>(send + off) & 15u) == 0;
      const size_t units = (hi - lo + 15) / 16;
      const size_t nthr = blockDim.x;
      size_t i = threadIdx.x;
      if (al) {
        for (; i + (kUnroll - 1) * nthr < units && lo + (i + (kUnroll - 1) * nthr) * 16 + 16 <= m;
             i += kUnroll * nthr) {
          uint4 v[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; u++) v[u] = ldCG(send + off + lo + (i + u * nthr) * 16);
#pragma unroll
          for (int u = 0; u < kUnroll; u++) multimemStore16(c.mcData + hoff + lo + (i + u * nthr) * 16, v[u]);
        }
      }
      for (; i < units; i += nthr) {
        const size_t u0 = lo + i * 16;
        uint4 v;
        if (al && u0 + 16 <= m) {
          v = ldCG(send + off + u0);
        } else {
          union { uint4 q; unsigned char b[16]; } t;
          t.q = make_uint4(0, 0, 0, 0);
          for (int j = 0; j < 16 && u0 + j < m; j++) t.b[j] = static_cast<unsigned char>(send[off + u0 + j]);
          v = t.q;
        }
        multimemStore16(c.mcData + hoff + u0, v);
      }
    }
    fenceProxyAlias();
    if (!blockBarrier(c, blk, kWhereGather)) return;
    if (lo < hi && !(me == root && recv == send)) copyAny(recv + off + lo, c.data[me] + hoff + lo, hi - lo);
  }
}

// ---------------------------------------------------------------------------
// Point-to-point: flow-controlled slot rings, one block per (peer, dir, ch).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) p2pKernel(DevComm c, P2pPlan plan) {
  const P2pWork w = plan.work[blockIdx.x];
  const int me = c.rank;
  __shared__ uint64_t sSeq;
  __shared__ int sFail;
  for (int j = 0; j < plan.nops; j++) {
    const P2pOpDesc op = plan.ops[j];
    if (op.kind != w.kind || (w.kind != kP2pCopy && op.peer != w.peer)) continue;
    const int nch = (w.kind == kP2pCopy) ? kMaxChannels : p2pChannels(op.bytes);
    if (w.ch >= nch) continue;
    size_t lo, hi;
    blockRange(op.bytes, nch, w.ch, 16, &lo, &hi);
    const size_t len = hi - lo;
    if (w.kind == kP2pCopy) {
      copyAny(op.dst + lo, op.src + lo, len);
      continue;
    }
    const size_t nchunks = (len + kP2pSlotBytes - 1) / kP2pSlotBytes;
    const int peer = op.peer;
    const int idx = peer * kMaxChannels + w.ch;  // my counters about `peer`
    const int ridx = me * kMaxChannels + w.ch;   // peer's counters about me
    if (threadIdx.x == 0) {
      sSeq = w.kind == kP2pSend ? ctrlAt<uint64_t>(c, me, kP2pSentOff)[idx] : ctrlAt<uint64_t>(c, me, kP2pRecvdOff)[idx];
      sFail = 0;
    }
    __syncthreads();
    const uint64_t base = sSeq;
    for (size_t q = 0; q < nchunks; q++) {
      const uint64_t seq = base + q;
      const size_t clen = (len - q * kP2pSlotBytes) < kP2pSlotBytes ? (len - q * kP2pSlotBytes) : kP2pSlotBytes;
      if (w.kind == kP2pSend) {
        char* ring = c.ctrl[peer] + kP2pOff + static_cast<size_t>(ridx) * kP2pSlots * kP2pSlotBytes;
        if (threadIdx.x == 0 && seq >= static_cast<uint64_t>(kP2pSlots)) {
          if (!waitAtLeast64(c, ctrlAt<uint64_t>(c, me, kP2pTailOff) + idx, seq - kP2pSlots + 1, kWhereP2pSend,
                             peer))
            sFail = 1;
        }
        __syncthreads();
        if (sFail) return;
        copyAny(ring + (seq % kP2pSlots) * kP2pSlotBytes, op.src + lo + q * kP2pSlotBytes, clen);
        __syncthreads();
        if (threadIdx.x == 0) {
          fenceSys();
          stReleaseSys64(ctrlAt<uint64_t>(c, peer, kP2pHeadOff) + ridx, seq + 1);
        }
      } else {
        const char* ring = c.ctrl[me] + kP2pOff + static_cast<size_t>(idx) * kP2pSlots * kP2pSlotBytes;
        if (threadIdx.x == 0) {
          if (!waitAtLeast64(c, ctrlAt<uint64_t>(c, me, kP2pHeadOff) + idx, seq + 1, kWhereP2pRecv, peer))
            sFail = 1;
        }
        __syncthreads();
        if (sFail) return;
        copyAny(op.dst + lo + q * kP2pSlotBytes, ring + (seq % kP2pSlots) * kP2pSlotBytes, clen);
        __syncthreads();
        if (threadIdx.x == 0) {
          fenceSys();
          stReleaseSys64(ctrlAt<uint64_t>(c, peer, kP2pTailOff) + ridx, seq + 1);
        }
      }
    }
    if (threadIdx.x == 0) {
      if (w.kind == kP2pSend)
        ctrlAt<uint64_t>(c, me, kP2pSentOff)[idx] = base + nchunks;
      else
        ctrlAt<uint64_t>(c, me, kP2pRecvdOff)[idx] = base + nchunks;
    }
    __syncthreads();
  }
}

}  // namespace dev
}  // namespace vccl
