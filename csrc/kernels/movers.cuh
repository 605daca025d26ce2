// SPDX-License-Identifier: Apache-2.0
// Block-level data movers with deep memory-level parallelism: the device
// counterparts of the reference's host reduction and scaling helpers
// (reference: src/core/reduce.cc:234-408, cpuReduce / cpuScaledAccumulate /
// cpuScaleCopy / cpuScale), with PreMulSum scaling fused into the load and
// average scaling into the store.
//
// NVLink loads take on the order of a microsecond to return, so a block
// that keeps one 16-byte load per thread in flight moves only ~8 KiB per
// round trip.  Every mover here issues kUnroll independent 16-byte loads
// per thread before consuming any of them.
#pragma once

#include <stdint.h>

#include "kernels/device_common.cuh"
#include "kernels/dtypes.cuh"

namespace vccl {
namespace dev {

constexpr int kUnroll = 8;

// Every mover takes the calling thread's index `tid` among the `nthr`
// threads that share the work; the short forms use the whole block.  A
// kernel that splits its warps into roles passes each role's own range.

// n16 16-byte units, dst and src 16-byte aligned.
__device__ __forceinline__ void copy16(char* dst, const char* src, size_t n16, size_t tid, size_t nthr) {
  size_t i = tid;
  for (; i + (kUnroll - 1) * nthr < n16; i += kUnroll * nthr) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; u++) v[u] = ldCG(src + (i + u * nthr) * 16);
#pragma unroll
    for (int u = 0; u < kUnroll; u++) stG(dst + (i + u * nthr) * 16, v[u]);
  }
  for (; i < n16; i += nthr) stG(dst + i * 16, ldCG(src + i * 16));
}

__device__ __forceinline__ void copy16(char* dst, const char* src, size_t n16) {
  copy16(dst, src, n16, threadIdx.x, blockDim.x);
}

// Byte copy choosing the widest access the alignment allows.
__device__ __forceinline__ void copyAny(char* dst, const char* src, size_t n, size_t tid, size_t nthr) {
  if (n == 0 || dst == src) return;
  const uintptr_t al = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
  if ((al & 15u) == 0) {
    copy16(dst, src, n / 16, tid, nthr);
    for (size_t i = n / 16 * 16 + tid; i < n; i += nthr) dst[i] = src[i];
  } else if ((al & 3u) == 0) {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    for (size_t i = tid; i < n / 4; i += nthr) d[i] = s[i];
    for (size_t i = n / 4 * 4 + tid; i < n; i += nthr) dst[i] = src[i];
  } else {
    for (size_t i = tid; i < n; i += nthr) dst[i] = src[i];
  }
}
__device__ __forceinline__ void copyAny(char* dst, const char* src, size_t n) {
  copyAny(dst, src, n, threadIdx.x, blockDim.x);
}

// dst[i] = src[i] * s (PreMulSum contribution) for `elems` elements.
template <typename T, bool VEC>
__device__ __forceinline__ void copyScaled(char* dst, const char* src, size_t elems, bool doScale, double s,
                                           size_t tid, size_t nthr) {
  if (!doScale) {
    if constexpr (VEC) {
      copy16(dst, src, elems * sizeof(T) / 16, tid, nthr);
      const size_t done = elems * sizeof(T) / 16 * 16 / sizeof(T);
      const T* sp = reinterpret_cast<const T*>(src);
      T* dp = reinterpret_cast<T*>(dst);
      for (size_t i = done + tid; i < elems; i += nthr) dp[i] = sp[i];
    } else {
      copyAny(dst, src, elems * sizeof(T), tid, nthr);
    }
    return;
  }
  size_t done = 0;
  if constexpr (VEC) {
    constexpr int N = 16 / sizeof(T);
    const size_t packs = elems / N;
    size_t i = tid;
    for (; i + (kUnroll - 1) * nthr < packs; i += kUnroll * nthr) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; u++) v[u] = ldCG(src + (i + u * nthr) * 16);
#pragma unroll
      for (int u = 0; u < kUnroll; u++) stG(dst + (i + u * nthr) * 16, scaledRaw<T>(v[u], true, s));
    }
    for (; i < packs; i += nthr) stG(dst + i * 16, scaledRaw<T>(ldCG(src + i * 16), true, s));
    done = packs * N;
  }
  const T* sp = reinterpret_cast<const T*>(src);
  T* dp = reinterpret_cast<T*>(dst);
  for (size_t i = done + tid; i < elems; i += nthr) dp[i] = scaledElem<T>(sp[i], true, s);
}
template <typename T, bool VEC>
__device__ __forceinline__ void copyScaled(char* dst, const char* src, size_t elems, bool doScale, double s) {
  copyScaled<T, VEC>(dst, src, elems, doScale, s, threadIdx.x, blockDim.x);
}

// out[i] = fold(own[i] * premul?, slots[p][i] for p != me) * (1/n if avg).
// `slot(p)` returns the base of source p's elements.
template <typename T, int K, bool VEC, typename SlotFn>
__device__ __forceinline__ void reduceInto(int n, int me, char* out, char* out2, const char* own, SlotFn slot,
                                           size_t elems, bool premul, double scalar, bool avg) {
  size_t done = 0;
  if constexpr (VEC) {
    constexpr int N = 16 / sizeof(T);
    constexpr int U = 4;
    const size_t packs = elems / N;
    const size_t nthr = blockDim.x;
    size_t i = threadIdx.x;
    for (; i + (U - 1) * nthr < packs; i += U * nthr) {
      Pack<T> acc[U];
      uint4 raw[U];
#pragma unroll
      for (int u = 0; u < U; u++) raw[u] = ldCG(own + (i + u * nthr) * 16);
#pragma unroll
      for (int u = 0; u < U; u++) {
        acc[u].load(raw[u]);
        if (premul) acc[u].scale(scalar);
      }
#pragma unroll 1
      for (int k = 1; k < n; k++) {
        int p = me + k;
        if (p >= n) p -= n;
        const char* sp = slot(p);
#pragma unroll
        for (int u = 0; u < U; u++) raw[u] = ldCG(sp + (i + u * nthr) * 16);
#pragma unroll
        for (int u = 0; u < U; u++) acc[u].template fold<K>(raw[u]);
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        if (avg) acc[u].scale(1.0 / n);
        const uint4 r = acc[u].pack();
        if (out) stG(out + (i + u * nthr) * 16, r);
        if (out2) stG(out2 + (i + u * nthr) * 16, r);
      }
    }
    for (; i < packs; i += nthr) {
      Pack<T> acc;
      acc.load(ldCG(own + i * 16));
      if (premul) acc.scale(scalar);
      for (int k = 1; k < n; k++) {
        int p = me + k;
        if (p >= n) p -= n;
        acc.template fold<K>(ldCG(slot(p) + i * 16));
      }
      if (avg) acc.scale(1.0 / n);
      const uint4 r = acc.pack();
      if (out) stG(out + i * 16, r);
      if (out2) stG(out2 + i * 16, r);
    }
    done = packs * N;
  }
  using E = Elem<T>;
  const T* op = reinterpret_cast<const T*>(own);
  for (size_t i = done + threadIdx.x; i < elems; i += blockDim.x) {
    typename E::Acc acc = E::toAcc(op[i]);
    if (premul) acc = scaleAcc<T>(acc, scalar);
    for (int k = 1; k < n; k++) {
      int p = me + k;
      if (p >= n) p -= n;
      acc = combine<T, K>(acc, E::toAcc(reinterpret_cast<const T*>(slot(p))[i]));
    }
    if (avg) acc = scaleAcc<T>(acc, 1.0 / n);
    const T r = E::fromAcc(acc);
    if (out) reinterpret_cast<T*>(out)[i] = r;
    if (out2) reinterpret_cast<T*>(out2)[i] = r;
  }
}

}  // namespace dev
}  // namespace vccl
