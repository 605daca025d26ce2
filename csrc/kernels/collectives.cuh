// SPDX-License-Identifier: Apache-2.0
// Reduction collectives over symmetric NVLink-mapped workspaces.
//
// These replace the reference's host-side ring / recursive-doubling / chain
// algorithms over TCP (reference: src/core/collectives.cc:102-620) with
// single-kernel algorithms that fit a uniform NVSwitch fabric:
//
//   allReduceLL       one NVLink hop: every rank stores its (pre-scaled)
//                     payload into every peer's LL region as 16-byte lines
//                     {data, flag, data, flag}; readers spin on the flags.
//                     No barriers.  Small messages.
//   allReduceTwoShot  push reduce-scatter into the owners' staging slots,
//                     local reduction, then every rank pulls the reduced
//                     chunks (also used for Reduce, where only the root
//                     pulls).  Any dtype/op.
//   allReduceNvls     copy into the multicast-bound staging region, then
//                     multimem.ld_reduce + multimem.st of the owned chunk
//                     (the NVSwitch reduces and broadcasts), copy out.
//   reduceScatterPush push chunk q to rank q's slot, reduce locally.
//
// Every barrier-based kernel begins with a barrier: once block b has met
// every peer in this launch, each peer has finished all earlier launches on
// this communicator, so staging memory may be overwritten.  Rounds inside a
// launch alternate staging halves or are separated by the data-ready
// barrier of the next round.
#pragma once

#include "kernels/coll_abi.cuh"
#include "kernels/device_common.cuh"
#include "kernels/dtypes.cuh"
#include "kernels/movers.cuh"
#include "kernels/ranges.cuh"

namespace vccl {
namespace dev {


// ---------------------------------------------------------------------------
// LL one-shot all-reduce.  Grid is always the communicator's llBlocks so every block's epoch
// advances once per launch (epochs are equal across blocks and ranks).
// send/recv must be 8-byte aligned and count*sizeof(T) <= kLLMaxBytes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t readWord(const char* base, size_t w, size_t bytes) {
  const size_t off = w * 8;
  if (off + 8 <= bytes) return *reinterpret_cast<const uint64_t*>(base + off);
  uint64_t v = 0;
  for (size_t i = 0; off + i < bytes; i++)
    v |= static_cast<uint64_t>(static_cast<unsigned char>(base[off + i])) << (8 * i);
  return v;
}
__device__ __forceinline__ void writeWord(char* base, size_t w, size_t bytes, uint64_t v) {
  const size_t off = w * 8;
  if (off + 8 <= bytes) {
    *reinterpret_cast<uint64_t*>(base + off) = v;
    return;
  }
  for (size_t i = 0; off + i < bytes; i++) base[off + i] = static_cast<char>((v >> (8 * i)) & 0xff);
}

template <typename T>
struct WordPack {
  static constexpr int N = 8 / sizeof(T);
  using Acc = typename Elem<T>::Acc;
  Acc v[N];
  __device__ __forceinline__ void load(uint64_t raw) {
    union { uint64_t u; T e[N]; } c;
    c.u = raw;
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = Elem<T>::toAcc(c.e[i]);
  }
  __device__ __forceinline__ uint64_t pack() const {
    union { uint64_t u; T e[N]; } c;
#pragma unroll
    for (int i = 0; i < N; i++) c.e[i] = Elem<T>::fromAcc(v[i]);
    return c.u;
  }
  template <int K>
  __device__ __forceinline__ void fold(uint64_t raw) {
    union { uint64_t u; T e[N]; } c;
    c.u = raw;
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = combine<T, K>(v[i], Elem<T>::toAcc(c.e[i]));
  }
  __device__ __forceinline__ void scale(double s) {
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = scaleAcc<T>(v[i], s);
  }
};

__device__ __forceinline__ void stVolatile16(char* p, const uint4& v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ldVolatile16(const char* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ char* llSlot(const DevComm& c, int owner, uint32_t parity, int src) {
  return c.ctrl[owner] + kLLOff + (static_cast<size_t>(parity) * kMaxRanks + src) * kLLSlotBytes;
}

// ---------------------------------------------------------------------------
// Two-shot all-reduce / reduce.  Staging: n input slots + 1 result slot of
// slotElems elements each.  root < 0: all-reduce; else only root gathers.
// ---------------------------------------------------------------------------
template <typename T, int K, bool VEC>
__global__ void __launch_bounds__(512) allReduceTwoShot(DevComm c, CollArgs a, size_t slotElems) {
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  constexpr size_t PK = VEC ? 16 / sizeof(T) : 1;
  const size_t esz = sizeof(T);
  const size_t slotBytes = slotElems * esz;
  if (!blockBarrier(c, blk, kWhereStart)) return;
  const size_t roundElems = slotElems * n;
  // Chunk size and block split are fixed for the launch (a short last
  // round is clipped, not re-split), so every block keeps its own slots.
  const size_t first = a.count < roundElems ? a.count : roundElems;
  const size_t ce = rankChunk(first, n, PK);
  size_t s0, s1;
  blockRange(ce, G, blk, PK, &s0, &s1);
  for (size_t base = 0; base < a.count; base += roundElems) {
    const size_t m = (a.count - base) < roundElems ? (a.count - base) : roundElems;
    // 1. push my contribution to chunk q into rank q's slot `me`
    for (int k = 1; k < n; k++) {
      const int q = (me + k) % n;
      const size_t lo = q * ce + s0;
      const size_t hiRaw = q * ce + s1;
      const size_t hi = hiRaw < m ? hiRaw : m;
      if (lo < hi)
        copyScaled<T, VEC>(c.data[q] + me * slotBytes + s0 * esz, a.send + (base + lo) * esz, hi - lo, a.premul,
                           a.scalar);
    }
    if (!blockBarrier(c, blk, kWherePush)) return;
    // 2. reduce my chunk
    {
      const size_t lo = me * ce + s0;
      const size_t hiRaw = me * ce + s1;
      const size_t hi = hiRaw < m ? hiRaw : m;
      if (lo < hi) {
        char* resultSlot = c.data[me] + n * slotBytes + s0 * esz;
        char* out = nullptr;
        char* out2 = nullptr;
        if (a.root < 0) {
          out = a.recv + (base + lo) * esz;
          out2 = resultSlot;
        } else if (a.root == me) {
          out = a.recv + (base + lo) * esz;
        } else {
          out2 = resultSlot;
        }
        const char* slots = c.data[me] + s0 * esz;
        reduceInto<T, K, VEC>(
            n, me, out, out2, a.send + (base + lo) * esz, [&](int p) { return slots + p * slotBytes; }, hi - lo,
            a.premul, a.scalar, a.avg);
      }
    }
    if (!blockBarrier(c, blk, kWhereReduce)) return;
    // 3. gather the reduced chunks
    if (a.root < 0 || a.root == me) {
      for (int k = 1; k < n; k++) {
        const int q = (me + k) % n;
        const size_t lo = q * ce + s0;
        const size_t hiRaw = q * ce + s1;
        const size_t hi = hiRaw < m ? hiRaw : m;
        if (lo < hi)
          copyScaled<T, VEC>(a.recv + (base + lo) * esz, c.data[q] + n * slotBytes + s0 * esz, hi - lo, false,
                             1.0);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// NVLS all-reduce (f32 / bf16 / f16; sum, and min/max for 16-bit floats).
// ---------------------------------------------------------------------------
template <typename T, int K>
struct Multimem;

#define VCCL_MM(T, TNAME, OPNAME, KV)                                                                     \
  template <>                                                                                             \
  struct Multimem<T, KV> {                                                                                \
    __device__ __forceinline__ static uint4 ldReduce(const char* p) {                                     \
      uint4 v;                                                                                            \
      asm volatile("multimem.ld_reduce.relaxed.sys.global." OPNAME ".v4." TNAME " {%0,%1,%2,%3}, [%4];" \
                   : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)                                           \
                   : "l"(p)                                                                               \
                   : "memory");                                                                           \
      return v;                                                                                           \
    }                                                                                                     \
  };
VCCL_MM(float, "f32", "add", kSum)
VCCL_MM(__nv_bfloat16, "bf16x2", "add.acc::f32", kSum)
VCCL_MM(__half, "f16x2", "add.acc::f32", kSum)
VCCL_MM(__nv_bfloat16, "bf16x2", "min", kMin)
VCCL_MM(__half, "f16x2", "min", kMin)
VCCL_MM(__nv_bfloat16, "bf16x2", "max", kMax)
VCCL_MM(__half, "f16x2", "max", kMax)
#undef VCCL_MM

template <typename T, int K>
struct HasMultimem {
  static constexpr bool value = false;
};
template <> struct HasMultimem<float, kSum> { static constexpr bool value = true; };
template <> struct HasMultimem<__nv_bfloat16, kSum> { static constexpr bool value = true; };
template <> struct HasMultimem<__half, kSum> { static constexpr bool value = true; };
template <> struct HasMultimem<__nv_bfloat16, kMin> { static constexpr bool value = true; };
template <> struct HasMultimem<__half, kMin> { static constexpr bool value = true; };
template <> struct HasMultimem<__nv_bfloat16, kMax> { static constexpr bool value = true; };
template <> struct HasMultimem<__half, kMax> { static constexpr bool value = true; };

__device__ __forceinline__ void multimemStore16(char* p, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Copy `elems` elements with optional scaling; any alignment on the user side.
template <typename T>
__device__ __forceinline__ void copyInScaled(char* dst, const char* src, size_t elems, bool doScale, double s,
                                             size_t tid, size_t nthr) {
  if (!doScale) {
    copyAny(dst, src, elems * sizeof(T), tid, nthr);
  } else if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0) {
    copyScaled<T, true>(dst, src, elems, true, s, tid, nthr);
  } else {
    copyScaled<T, false>(dst, src, elems, true, s, tid, nthr);
  }
}
template <typename T>
__device__ __forceinline__ void copyInScaled(char* dst, const char* src, size_t elems, bool doScale, double s) {
  copyInScaled<T>(dst, src, elems, doScale, s, threadIdx.x, blockDim.x);
}

// Reduce bytes [lo, hi) of the multicast source through the switch and store
// the result to the same bytes of the multicast destination, i.e. of every
// rank's copy (16-byte units, U in flight per thread; the last unit is
// rounded up to 16 bytes).
template <typename T, int K, int U = 4>
__device__ __forceinline__ void nvlsReduceRange(const char* mcSrc, char* mcDst, size_t lo, size_t hi, bool avg,
                                                int n, size_t tid, size_t nthr) {
  const size_t units = (hi - lo + 15) / 16;
  size_t i = tid;
  for (; i + (U - 1) * nthr < units; i += U * nthr) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) v[u] = Multimem<T, K>::ldReduce(mcSrc + lo + (i + u * nthr) * 16);
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (avg) {
        Pack<T> p;
        p.load(v[u]);
        p.scale(1.0 / n);
        v[u] = p.pack();
      }
      multimemStore16(mcDst + lo + (i + u * nthr) * 16, v[u]);
    }
  }
  // Fewer than U * nthr units remain: one guarded batch keeps every
  // thread's remaining loads in flight together.
  if (i < units) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      if (i + u * nthr < units) v[u] = Multimem<T, K>::ldReduce(mcSrc + lo + (i + u * nthr) * 16);
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (i + u * nthr >= units) break;
      if (avg) {
        Pack<T> p;
        p.load(v[u]);
        p.scale(1.0 / n);
        v[u] = p.pack();
      }
      multimemStore16(mcDst + lo + (i + u * nthr) * 16, v[u]);
    }
  }
}
// In place: the staging region is both source and destination.
template <typename T, int K, int U = 4>
__device__ __forceinline__ void nvlsReduceRange(char* mc, size_t lo, size_t hi, bool avg, int n, size_t tid,
                                                size_t nthr) {
  nvlsReduceRange<T, K, U>(mc, mc, lo, hi, avg, n, tid, nthr);
}
template <typename T, int K>
__device__ __forceinline__ void nvlsReduceRange(char* mc, size_t lo, size_t hi, bool avg, int n) {
  nvlsReduceRange<T, K>(mc, mc, lo, hi, avg, n, threadIdx.x, blockDim.x);
}

template <typename T, int K>
__global__ void __launch_bounds__(512) allReduceNvls(DevComm c, CollArgs a, size_t roundBytes) {
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  const size_t esz = sizeof(T);
  const size_t total = a.count * esz;
  if (!blockBarrier(c, blk, kWhereStart)) return;
  char* local = c.data[me];
  // One chunk size for every round of the launch (see roundRange).
  const size_t cb = nvlsRoundChunk(total, n, roundBytes);
  const size_t step = cb * n;
  size_t s0, s1;
  blockRange(cb, G, blk, 16, &s0, &s1);
  for (size_t off = 0; off < total; off += step) {
    const size_t m = (total - off) < step ? (total - off) : step;
    // 1. copy in: my sub-slice of every chunk
    for (int q = 0; q < n; q++) {
      const size_t lo = q * cb + s0;
      const size_t hiRaw = q * cb + s1;
      const size_t hi = hiRaw < m ? hiRaw : m;
      if (lo < hi) copyInScaled<T>(local + lo, a.send + off + lo, (hi - lo) / esz, a.premul, a.scalar);
    }
    // The copy-in wrote through this GPU's own address; the peers read it
    // through the multicast address (another alias of the same memory).
    fenceProxyAlias();
    if (!blockBarrier(c, blk, kWhereNvls)) return;
    // 2. reduce my chunk through the switch and broadcast the result
    if constexpr (HasMultimem<T, K>::value) {
      const size_t lo = me * cb + s0;
      const size_t hiRaw = me * cb + s1;
      const size_t hi = hiRaw < m ? hiRaw : m;
      if (lo < hi) nvlsReduceRange<T, K>(c.mcData, lo, hi, a.avg != 0, n);
    }
    fenceProxyAlias();
    if (!blockBarrier(c, blk, kWhereNvls)) return;
    // 3. copy out
    for (int q = 0; q < n; q++) {
      const size_t lo = q * cb + s0;
      const size_t hiRaw = q * cb + s1;
      const size_t hi = hiRaw < m ? hiRaw : m;
      if (lo < hi) copyAny(a.recv + off + lo, local + lo, hi - lo);
    }
  }
}

// ---------------------------------------------------------------------------
// Pipelined NVLS all-reduce.  The message is cut into pieces of n * cb bytes
// (cb per rank chunk, a multiple of 16) that rotate through kPipeSlots
// staging slots of slotBytes.  Step s copies piece s in, reduces piece s-1
// through the switch and copies piece s-2 out, each with its own warps, and
// then meets the peers once, so the HBM copies of one piece overlap the
// NVLink traffic of the next.  Block b owns the same bytes
// [q*cb + s0, q*cb + s1) of every slot for every piece, so blocks never
// touch each other's staging, and the barrier after each step orders block
// b's uses of a slot across ranks:
//   reduce(p)   at step p+1 reads what every rank copied in at step p,
//   copy-out(p) at step p+2 reads what the owners stored at step p+1,
//   copy-in(p+3) at step p+3 refills the slot after both.
// The three uses within a step are on three different slots.
// Warps [0, kPipeInWarps) copy in, the next kPipeRedWarps reduce, the rest
// (of the 16 launched) copy out.
// ---------------------------------------------------------------------------
constexpr int kPipeSlots = 3;
constexpr int kPipeInWarps = 4;
constexpr int kPipeRedWarps = 8;
constexpr int kPipeThreads = 512;

template <typename T, int K>
__global__ void __launch_bounds__(kPipeThreads) allReduceNvlsPipe(DevComm c, CollArgs a, size_t cb,
                                                                  size_t slotBytes) {
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  const size_t esz = sizeof(T);
  const size_t total = a.count * esz;
  const size_t piece = cb * n;
  const size_t P = (total + piece - 1) / piece;
  const int warp = static_cast<int>(threadIdx.x) / 32;
  const int role = warp < kPipeInWarps ? 0 : (warp < kPipeInWarps + kPipeRedWarps ? 1 : 2);
  const int roleBase = role == 0 ? 0 : (role == 1 ? kPipeInWarps : kPipeInWarps + kPipeRedWarps);
  const int roleWarps = role == 0 ? kPipeInWarps : (role == 1 ? kPipeRedWarps : 16 - kPipeInWarps - kPipeRedWarps);
  const size_t tid = threadIdx.x - roleBase * 32;
  const size_t nthr = static_cast<size_t>(roleWarps) * 32;
  size_t s0, s1;
  blockRange(cb, G, blk, 16, &s0, &s1);
  if (!blockBarrier(c, blk, kWhereStart)) return;
  char* local = c.data[me];
  for (size_t st = 0; st < P + 2; st++) {
    if (role == 0 && st < P) {
      const size_t off = st * piece;
      const size_t m = (total - off) < piece ? (total - off) : piece;
      char* slot = local + (st % kPipeSlots) * slotBytes;
      for (int q = 0; q < n; q++) {
        const size_t lo = q * cb + s0;
        const size_t hiRaw = q * cb + s1;
        const size_t hi = hiRaw < m ? hiRaw : m;
        if (lo < hi) copyInScaled<T>(slot + lo, a.send + off + lo, (hi - lo) / esz, a.premul, a.scalar, tid, nthr);
      }
    } else if (role == 1 && st >= 1 && st <= P) {
      if constexpr (HasMultimem<T, K>::value) {
        const size_t p = st - 1;
        const size_t off = p * piece;
        const size_t m = (total - off) < piece ? (total - off) : piece;
        const size_t lo = me * cb + s0;
        const size_t hiRaw = me * cb + s1;
        const size_t hi = hiRaw < m ? hiRaw : m;
        if (lo < hi)
          nvlsReduceRange<T, K, 8>(c.mcData + (p % kPipeSlots) * slotBytes, lo, hi, a.avg != 0, n, tid, nthr);
      }
    } else if (role == 2 && st >= 2) {
      const size_t p = st - 2;
      const size_t off = p * piece;
      const size_t m = (total - off) < piece ? (total - off) : piece;
      const char* slot = local + (p % kPipeSlots) * slotBytes;
      for (int q = 0; q < n; q++) {
        const size_t lo = q * cb + s0;
        const size_t hiRaw = q * cb + s1;
        const size_t hi = hiRaw < m ? hiRaw : m;
        if (lo < hi) copyAny(a.recv + off + lo, slot + lo, hi - lo, tid, nthr);
      }
    }
    if (st == P + 1) break;  // the last step only copies out
    fenceProxyAlias();
    if (!blockBarrier(c, blk, kWhereNvls)) return;
  }
}

// ---------------------------------------------------------------------------
// Reduce-scatter: push chunk q to rank q's slot, reduce locally.
// ---------------------------------------------------------------------------
template <typename T, int K, bool VEC>
__global__ void __launch_bounds__(512) reduceScatterPush(DevComm c, CollArgs a, size_t slotElems) {
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  constexpr size_t PK = VEC ? 16 / sizeof(T) : 1;
  const size_t esz = sizeof(T);
  const size_t slotBytes = slotElems * esz;
  const size_t half = (c.dataBytes / 2) / 16 * 16;
  if (!blockBarrier(c, blk, kWhereStart)) return;
  const size_t rc = a.count;
  int k = 0;
  const size_t full = rc < slotElems ? rc : slotElems;
  for (size_t base = 0; base < rc; base += slotElems, k++) {
    const size_t m = (rc - base) < slotElems ? (rc - base) : slotElems;
    size_t s0, s1;
    roundRange(full, m, G, blk, PK, &s0, &s1);
    const size_t hoff = (k & 1) * half;
    if (s0 < s1) {
      for (int s = 1; s < n; s++) {
        const int q = (me + s) % n;
        copyScaled<T, VEC>(c.data[q] + hoff + me * slotBytes + s0 * esz, a.send + (q * rc + base + s0) * esz,
                           s1 - s0, a.premul, a.scalar);
      }
    }
    if (!blockBarrier(c, blk, kWherePush)) return;
    if (s0 < s1) {
      const char* slots = c.data[me] + hoff + s0 * esz;
      reduceInto<T, K, VEC>(
          n, me, a.recv + (base + s0) * esz, nullptr, a.send + (me * rc + base + s0) * esz,
          [&](int p) { return slots + p * slotBytes; }, s1 - s0, a.premul, a.scalar, a.avg);
    }
  }
}

}  // namespace dev
}  // namespace vccl

#include "kernels/ll.cuh"
