// SPDX-License-Identifier: Apache-2.0
// LL ("low latency") kernels: data travels as 16-byte lines
// {data32, flag, data32, flag} whose flags carry the launch epoch, so a
// reader needs no barrier and no fence — it spins until both flags of a
// line match.  NVLink delivers each 8-byte half atomically, which is all
// the protocol relies on.
//
// Every LL kernel runs with the communicator's LL grid (llBlocks) and bumps each block's
// epoch once, so epochs agree across blocks, ranks and kernel kinds.  A slot
// of parity p is rewritten two LL launches later; that is safe because in
// every LL launch each rank receives from every other rank, so finishing
// launch k+1 proves every peer has finished launch k.
//
// Loads and stores are batched kLLUnroll deep per thread: an LL kernel is
// otherwise bound by one outstanding memory operation per thread.
//
// These replace the reference's latency path for small messages, the
// recursive-doubling all-gather / all-reduce below its RD_MAX thresholds
// (reference: src/core/collectives.cc:156-184, :359-400): NVSwitch gives
// every pair full bandwidth, so one hop to every peer beats a log-step tree.
//
// Included at the end of collectives.cuh.
#pragma once

namespace vccl {
namespace dev {

constexpr int kLLUnroll = 4;

__device__ __forceinline__ char* llResSlot(const DevComm& c, int owner, uint32_t parity, int src) {
  return c.ctrl[owner] + kLLResOff + (static_cast<size_t>(parity) * kMaxRanks + src) * kLLSlotBytes;
}

// Epochs run 1, 2, ..., 2^32 - 1, then 2, 3, ...: they never take the
// value 0 the slots are filled with at set-up (a line no peer has written
// yet can never look current, even after the counter wraps), and the wrap
// keeps odd and even epochs alternating, so a slot of one parity is still
// rewritten only every second launch.
__device__ __forceinline__ uint32_t llEpoch(const DevComm& c) {
  __shared__ uint32_t sE;
  if (threadIdx.x == 0) {
    uint32_t* ep = ctrlAt<uint32_t>(c, c.rank, kLLEpochOff) + blockIdx.x;
    sE = *ep + 1u;
    if (sE == 0u) sE = 2u;
    *ep = sE;
  }
  __syncthreads();
  return sE;
}

__device__ __forceinline__ uint4 llLine(uint64_t word, uint32_t e) {
  return make_uint4(static_cast<uint32_t>(word), e, static_cast<uint32_t>(word >> 32), e);
}

__device__ __forceinline__ void llPut(const DevComm& c, int peer, uint32_t par, uint32_t e, size_t w,
                                      uint64_t word) {
  stVolatile16(llSlot(c, peer, par, c.rank) + w * 16, llLine(word, e));
}

// Spin on one line until both flags equal e (bounded).
__device__ __forceinline__ bool llSpin(const DevComm& c, const char* p, uint32_t e, uint4* v) {
  const uint64_t start = globalTimerNs();
  for (uint32_t spin = 1;; ++spin) {
    *v = ldVolatile16(p);
    if (v->y == e && v->w == e) return true;
    if ((spin & 1023u) == 0u && shouldGiveUp(c, start, kWhereLL, 0)) return false;
  }
}

__device__ __forceinline__ bool llWait(const DevComm& c, const char* p, uint32_t e, uint64_t* out) {
  uint4 v = ldVolatile16(p);
  if ((v.y != e || v.w != e) && !llSpin(c, p, e, &v)) return false;
  *out = static_cast<uint64_t>(v.x) | (static_cast<uint64_t>(v.z) << 32);
  return true;
}

// Wait for lines i0 + u*stride (u < U, index < lim) of `slot`.
template <int U>
__device__ __forceinline__ bool llWaitU(const DevComm& c, const char* slot, size_t i0, size_t stride, size_t lim,
                                        uint32_t e, uint64_t (&out)[U]) {
  uint4 v[U];
#pragma unroll
  for (int u = 0; u < U; u++) {
    const size_t i = i0 + u * stride;
    if (i < lim) v[u] = ldVolatile16(slot + i * 16);
  }
#pragma unroll
  for (int u = 0; u < U; u++) {
    const size_t i = i0 + u * stride;
    if (i < lim) {
      if ((v[u].y != e || v[u].w != e) && !llSpin(c, slot + i * 16, e, &v[u])) return false;
      out[u] = static_cast<uint64_t>(v[u].x) | (static_cast<uint64_t>(v[u].z) << 32);
    }
  }
  return true;
}

template <typename T>
__device__ __forceinline__ uint64_t scaledWord(uint64_t word, bool premul, double s) {
  if (!premul) return word;
  WordPack<T> p;
  p.load(word);
  p.scale(s);
  return p.pack();
}

// ---------------------------------------------------------------------------
// One-shot LL all-reduce: every rank stores its payload into every peer.
// send/recv 8-byte aligned, payload <= kLLMaxBytes.
// ---------------------------------------------------------------------------
template <typename T, int K>
__global__ void __launch_bounds__(512) allReduceLL(DevComm c, CollArgs a) {
  constexpr int U = kLLUnroll;
  const uint32_t e = llEpoch(c);
  const uint32_t par = e & 1u;
  const int n = c.nranks, me = c.rank;
  const size_t bytes = a.count * sizeof(T);
  const size_t words = (bytes + 7) / 8;
  const size_t nthr = blockDim.x;
  size_t w0, w1;
  blockRange(words, gridDim.x, blockIdx.x, 1, &w0, &w1);
  for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
    uint64_t word[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      if (b + u * nthr < w1) word[u] = scaledWord<T>(readWord(a.send, b + u * nthr, bytes), a.premul, a.scalar);
    for (int k = 1; k < n; k++) {
      char* dst = llSlot(c, (me + k) % n, par, me);
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) stVolatile16(dst + (b + u * nthr) * 16, llLine(word[u], e));
    }
  }
  for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
    WordPack<T> acc[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (b + u * nthr < w1) {
        acc[u].load(readWord(a.send, b + u * nthr, bytes));
        if (a.premul) acc[u].scale(a.scalar);
      }
    }
    for (int k = 1; k < n; k++) {
      uint64_t v[U];
      if (!llWaitU<U>(c, llSlot(c, me, par, (me + k) % n), b, nthr, w1, e, v)) return;
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) acc[u].template fold<K>(v[u]);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (b + u * nthr < w1) {
        if (a.avg) acc[u].scale(1.0 / n);
        writeWord(a.recv, b + u * nthr, bytes, acc[u].pack());
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Two-shot LL all-reduce: chunk q travels to rank q as LL lines, q reduces
// it and sends the result to every rank as LL lines.  Two hops, no barrier;
// per GPU it moves 4 (n-1)/n S each way against 2 (n-1) S for the one-shot.
// Chunk payload <= kLLMaxBytes.
// ---------------------------------------------------------------------------
template <typename T, int K>
__global__ void __launch_bounds__(512) allReduceLL2(DevComm c, CollArgs a) {
  constexpr int U = kLLUnroll;
  const uint32_t e = llEpoch(c);
  const uint32_t par = e & 1u;
  const int n = c.nranks, me = c.rank;
  const size_t bytes = a.count * sizeof(T);
  const size_t words = (bytes + 7) / 8;
  const size_t cw = (words + n - 1) / n;  // chunk size in words
  const size_t nthr = blockDim.x;
  size_t s0, s1;
  blockRange(cw, gridDim.x, blockIdx.x, 1, &s0, &s1);
  // Words of chunk q this block handles: [q*cw + s0, min(q*cw + s1, words)).
  auto chunkEnd = [&](int q) {
    const size_t e1 = q * cw + s1;
    return (e1 < words ? e1 : words) - q * cw;  // as chunk-local index limit
  };
  // 1. my contribution to every other chunk -> its owner
  for (int k = 1; k < n; k++) {
    const int q = (me + k) % n;
    const size_t lim = q * cw < words ? chunkEnd(q) : 0;
    char* dst = llSlot(c, q, par, me);
    for (size_t b = s0 + threadIdx.x; b < lim; b += U * nthr) {
      uint64_t word[U];
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < lim)
          word[u] = scaledWord<T>(readWord(a.send, q * cw + b + u * nthr, bytes), a.premul, a.scalar);
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < lim) stVolatile16(dst + (b + u * nthr) * 16, llLine(word[u], e));
    }
  }
  // 2. reduce my chunk, publish the result to everyone
  {
    const size_t lim = me * cw < words ? chunkEnd(me) : 0;
    for (size_t b = s0 + threadIdx.x; b < lim; b += U * nthr) {
      WordPack<T> acc[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        if (b + u * nthr < lim) {
          acc[u].load(readWord(a.send, me * cw + b + u * nthr, bytes));
          if (a.premul) acc[u].scale(a.scalar);
        }
      }
      for (int k = 1; k < n; k++) {
        uint64_t v[U];
        if (!llWaitU<U>(c, llSlot(c, me, par, (me + k) % n), b, nthr, lim, e, v)) return;
#pragma unroll
        for (int u = 0; u < U; u++)
          if (b + u * nthr < lim) acc[u].template fold<K>(v[u]);
      }
      uint64_t r[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        if (b + u * nthr < lim) {
          if (a.avg) acc[u].scale(1.0 / n);
          r[u] = acc[u].pack();
          writeWord(a.recv, me * cw + b + u * nthr, bytes, r[u]);
        }
      }
      for (int k = 1; k < n; k++) {
        char* dst = llResSlot(c, (me + k) % n, par, me);
#pragma unroll
        for (int u = 0; u < U; u++)
          if (b + u * nthr < lim) stVolatile16(dst + (b + u * nthr) * 16, llLine(r[u], e));
      }
    }
  }
  // 3. collect the other chunks
  for (int k = 1; k < n; k++) {
    const int q = (me + k) % n;
    const size_t lim = q * cw < words ? chunkEnd(q) : 0;
    const char* src = llResSlot(c, me, par, q);
    for (size_t b = s0 + threadIdx.x; b < lim; b += U * nthr) {
      uint64_t v[U];
      if (!llWaitU<U>(c, src, b, nthr, lim, e, v)) return;
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < lim) writeWord(a.recv, q * cw + b + u * nthr, bytes, v[u]);
    }
  }
}

// ---------------------------------------------------------------------------
// LL reduce-scatter: chunk q (recvcount elements) goes to rank q as LL
// lines; q folds them into its own chunk.  recvcount*sizeof(T) % 8 == 0 and
// <= kLLMaxBytes; send/recv 8-byte aligned.
// ---------------------------------------------------------------------------
template <typename T, int K>
__global__ void __launch_bounds__(512) reduceScatterLL(DevComm c, CollArgs a) {
  constexpr int U = kLLUnroll;
  const uint32_t e = llEpoch(c);
  const uint32_t par = e & 1u;
  const int n = c.nranks, me = c.rank;
  const size_t bytes = a.count * sizeof(T);
  const size_t words = bytes / 8;
  const size_t nthr = blockDim.x;
  size_t w0, w1;
  blockRange(words, gridDim.x, blockIdx.x, 1, &w0, &w1);
  for (int k = 1; k < n; k++) {
    const int q = (me + k) % n;
    char* dst = llSlot(c, q, par, me);
    const char* src = a.send + q * bytes;
    for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
      uint64_t word[U];
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1)
          word[u] = scaledWord<T>(*reinterpret_cast<const uint64_t*>(src + (b + u * nthr) * 8), a.premul, a.scalar);
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) stVolatile16(dst + (b + u * nthr) * 16, llLine(word[u], e));
    }
  }
  const char* own = a.send + me * bytes;
  for (size_t b = w0 + threadIdx.x; b < w1; b += U * nthr) {
    WordPack<T> acc[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (b + u * nthr < w1) {
        acc[u].load(*reinterpret_cast<const uint64_t*>(own + (b + u * nthr) * 8));
        if (a.premul) acc[u].scale(a.scalar);
      }
    }
    for (int k = 1; k < n; k++) {
      uint64_t v[U];
      if (!llWaitU<U>(c, llSlot(c, me, par, (me + k) % n), b, nthr, w1, e, v)) return;
#pragma unroll
      for (int u = 0; u < U; u++)
        if (b + u * nthr < w1) acc[u].template fold<K>(v[u]);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (b + u * nthr < w1) {
        if (a.avg) acc[u].scale(1.0 / n);
        *reinterpret_cast<uint64_t*>(a.recv + (b + u * nthr) * 8) = acc[u].pack();
      }
    }
  }
}

}  // namespace dev
}  // namespace vccl
