// SPDX-License-Identifier: Apache-2.0
// Expert-parallel MoE dispatch and combine over NVLink, with the dispatch
// fused with fp8 e4m3 1x128 block quantisation.
//
// The reference only has the all-to-all(v) primitive for this (reference:
// src/core/collectives.cc:708-740, :853-884, pairwise host exchanges).  Here
// the routing is done on the device and every token crosses NVLink once,
// already quantised:
//
//   dispatch  1. count   (1 CTA)  count the (token, slot) pairs for every
//                                 destination rank, give each pair its index
//                                 among this rank's pairs to that rank, and
//                                 exchange the counts so every rank knows the
//                                 whole rank x rank count matrix.  The
//                                 exchange also orders this call after every
//                                 peer's previous call (the receive region is
//                                 only rewritten once its reader is done).
//             2. push    (grid)   one warp per token: load the bf16 row once,
//                                 find each 128-element block's absolute max,
//                                 quantise to e4m3 (scale = amax / 448) and
//                                 store the fp8 row, its scales and routing
//                                 metadata straight into each destination's
//                                 receive region at its final row.
//             3. receive (grid)   wait for every source, then dequantise the
//                                 received rows into the caller's bf16 buffer.
//   combine   1. push    (grid)   one warp per received row: scale the expert
//                                 output by its routing weight and store it
//                                 into the source rank's slot (token, k).
//             2. reduce  (grid)   wait for every expert rank, then sum the k
//                                 slots of every token in fp32.
//
// Rows received by a rank are ordered by (source rank, token, k).  All
// synchronisation is device-side (flags and counters in the control
// region), so the calls are stream-ordered and host-free.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "common/log.h"
#include "common/trace.h"
#include "kernels/collectives.cuh"
#include "runtime/comm.h"
#include "vccl_tp.h"

namespace vccl {
namespace moe {

using dev::DevComm;

constexpr int kMaxTopk = 8;
constexpr int kGrid = 256;       // fixed grid of the push/receive/reduce kernels (block counters)
// The single-rank kernels keep no block counters, so their grid can fill
// the GPU: 4 blocks of 256 threads per SM, as many as the dispatch kernel's
// 64 registers per thread allow (the dispatch profile showed 22 % of the
// warp slots in use with kGrid, latency-bound).
constexpr int kLocalBlocksPerSm = 4;
constexpr int kThreads = 256;    // 8 warps
constexpr float kFp8Max = 448.0f;

// Byte offsets inside every rank's MoE region.  They depend only on
// (capacity, hidden), which every rank passes identically, so a sender can
// address a receiver's rows.
struct Layout {
  size_t rxData;   // fp8 [cap][H]
  size_t rxScale;  // f32 [cap][H/128]
  size_t rxMeta;   // int4 [cap]: source rank, source token, k, local expert
  size_t rxW;      // f32 [cap]: routing weight
  size_t comb;     // bf16 [cap][H]: combine slots (token * topk + k) of this rank's tokens
  size_t pairPos;  // int [cap]: index of each of my pairs among my pairs to its destination
  size_t info;     // Info
  size_t total;
};

struct Info {
  int offs[dev::kMaxRanks];     // first row of my pairs in each destination's region
  int totalAt[dev::kMaxRanks];  // rows routed to each destination (all sources)
  int recv;                     // rows this rank received (clamped to capacity)
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

Layout layoutFor(int cap, int H) {
  Layout L;
  const size_t c = static_cast<size_t>(cap);
  L.rxData = 0;
  L.rxScale = align256(c * H);
  L.rxMeta = L.rxScale + align256(c * (H / 128) * 4);
  L.rxW = L.rxMeta + align256(c * 16);
  L.comb = L.rxW + align256(c * 4);
  L.pairPos = L.comb + align256(c * H * 2);
  L.info = L.pairPos + align256(c * 4);
  L.total = L.info + 256;
  return L;
}

using dev::redAddReleaseSys;

__device__ __forceinline__ uint32_t* ctrl32(const DevComm& c, int rank, size_t off) {
  return dev::ctrlAt<uint32_t>(c, rank, off);
}

// The last of the grid's blocks to get here (counter `which`, one per kernel
// kind) returns true.  Counters count blocks over all calls; the grid is
// fixed, so call e (1-based) ends at e * gridDim.x.
__device__ __forceinline__ bool lastBlock(const DevComm& c, int which, uint32_t e) {
  const uint32_t old = atomicAdd(ctrl32(c, c.rank, dev::kMoeBlocksOff) + which, 1u);
  return old + 1u == e * gridDim.x;
}

__device__ __forceinline__ void unpackBf16x8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 p = __bfloat1622float2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ uint4 packBf16x8(const float (&f)[8]) {
  uint4 o;
  uint32_t* u = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    u[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return o;
}

// 8 floats -> 8 e4m3 bytes (round to nearest even, saturating at +-448).
__device__ __forceinline__ uint2 toFp8x8(const float (&f)[8]) {
  uint32_t w[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i], f[4 * i + 1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi =
        __nv_cvt_float2_to_fp8x2(make_float2(f[4 * i + 2], f[4 * i + 3]), __NV_SATFINITE, __NV_E4M3);
    w[i] = lo | (hi << 16);
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ void fromFp8x8(uint2 q, float (&f)[8]) {
  const uint32_t w[2] = {q.x, q.y};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>((w[i / 2] >> (16 * (i % 2))) & 0xffffu);
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

// Chunks of 256 elements (8 per lane) each warp keeps in flight per row.
constexpr int kChunkUnroll = 4;

// Load this lane's 16 bytes of kChunkUnroll consecutive 256-element chunks
// (zeros past the row end) before any of them is used.
__device__ __forceinline__ void loadChunks(const uint4* row, int c0, int H, int lane, uint4 (&raw)[kChunkUnroll]) {
#pragma unroll
  for (int u = 0; u < kChunkUnroll; u++) {
    const int col = c0 + u * 256 + lane * 8;
    raw[u] = col < H ? row[col / 8] : make_uint4(0, 0, 0, 0);
  }
}

// Quantise the 8 values of this lane; the 16 lanes of a half-warp share one
// 128-element block (all 32 lanes must call this).
__device__ __forceinline__ uint2 quantize8(float (&f)[8], bool active, float* scaleOut) {
  float amax = 0.0f;
  if (active) {
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(f[i]));
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = amax > 0.0f ? amax / kFp8Max : 1.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) f[i] = f[i] / scale;
  *scaleOut = scale;
  return toFp8x8(f);
}

// ---------------------------------------------------------------------------
// dispatch 1: counts, pair positions, count-matrix exchange
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) moeCount(DevComm c, const int* ids, int P, int epr, int numExperts, int cap,
                                                 Layout L, int* recvCount) {
  __shared__ uint32_t sE;
  __shared__ int sWarp[32][dev::kMaxRanks];
  __shared__ int sTot[dev::kMaxRanks];
  __shared__ int sFail;
  const int n = c.nranks, me = c.rank, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    sE = *ctrl32(c, me, dev::kMoeDispEpochOff) + 1u;
    sFail = 0;
  }
  __syncthreads();
  const uint32_t e = sE, par = e & 1u;
  char* base = c.moe[me];
  int* pairPos = reinterpret_cast<int*>(base + L.pairPos);
  Info* info = reinterpret_cast<Info*>(base + L.info);
  const int per = (P + 1023) / 1024;
  const int lo = min(P, tid * per), hi = min(P, lo + per);
  int cnt[dev::kMaxRanks];
#pragma unroll
  for (int d = 0; d < dev::kMaxRanks; d++) cnt[d] = 0;
  for (int i = lo; i < hi; i++) {
    const int id = ids[i];
    if (id >= 0 && id < numExperts) {
      const int d = id / epr;
#pragma unroll
      for (int q = 0; q < dev::kMaxRanks; q++) cnt[q] += (q == d);
    }
  }
  // Block-wide exclusive scan of the counts, one destination at a time.
  int excl[dev::kMaxRanks];
#pragma unroll
  for (int d = 0; d < dev::kMaxRanks; d++) {
    int x = cnt[d];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) sWarp[warp][d] = x;
    excl[d] = x - cnt[d];
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int d = 0; d < dev::kMaxRanks; d++) {
      const int v = sWarp[lane][d];
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      sWarp[lane][d] = x - v;
      if (lane == 31) sTot[d] = x;
    }
  }
  __syncthreads();
#pragma unroll
  for (int d = 0; d < dev::kMaxRanks; d++) excl[d] += sWarp[warp][d];
  for (int i = lo; i < hi; i++) {
    const int id = ids[i];
    int pos = -1;
    if (id >= 0 && id < numExperts) {
      const int d = id / epr;
#pragma unroll
      for (int q = 0; q < dev::kMaxRanks; q++)
        if (q == d) pos = excl[q]++;
    }
    pairPos[i] = pos;
  }
  // My row of the count matrix goes to every rank (me included).
  if (tid < n) {
    uint32_t* row = ctrl32(c, tid, dev::kMoeCountsOff) + (par * dev::kMaxRanks + me) * 16;
    for (int d = 0; d < n; d++) dev::stRelaxedSys(row + 1 + d, static_cast<uint32_t>(sTot[d]));
    dev::stReleaseSys32(row, e);
  }
  if (tid < n) {
    const uint32_t* row = ctrl32(c, me, dev::kMoeCountsOff) + (par * dev::kMaxRanks + tid) * 16;
    if (!dev::waitAcquire(c, row, e, dev::kWhereMoe, tid, 32)) sFail = 1;
  }
  __syncthreads();
  if (tid == 0) {
    dev::fenceSys();
    const volatile uint32_t* rows = ctrl32(c, me, dev::kMoeCountsOff) + par * dev::kMaxRanks * 16;
    for (int d = 0; d < dev::kMaxRanks; d++) {
      int off = 0, tot = 0;
      for (int s = 0; s < n && d < n && !sFail; s++) {
        const int v = static_cast<int>(rows[s * 16 + 1 + d]);
        if (s < me) off += v;
        tot += v;
      }
      info->offs[d] = off;
      info->totalAt[d] = tot;
    }
    int recv = sFail ? 0 : info->totalAt[me];
    if (recv > cap) {
      dev::recordFailure(c, dev::kErrCapacity, dev::kWhereMoe, static_cast<uint32_t>(recv));
      recv = cap;
    }
    info->recv = recv;
    *recvCount = recv;
  }
}

// ---------------------------------------------------------------------------
// dispatch 2: quantise and push
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) moePush(DevComm c, const __nv_bfloat16* x, const int* ids, const float* w,
                                                    int T, int H, int topk, int epr, int numExperts, int cap,
                                                    Layout L) {
  __shared__ uint32_t sE;
  if (threadIdx.x == 0) sE = *ctrl32(c, c.rank, dev::kMoeDispEpochOff) + 1u;
  __syncthreads();
  const uint32_t e = sE;
  const int n = c.nranks, me = c.rank;
  const char* base = c.moe[me];
  const int* pairPos = reinterpret_cast<const int*>(base + L.pairPos);
  const Info* info = reinterpret_cast<const Info*>(base + L.info);
  const int lane = threadIdx.x & 31;
  const int nb = H / 128;
  const int gw = blockIdx.x * (kThreads / 32) + threadIdx.x / 32, nw = gridDim.x * (kThreads / 32);
  for (int t = gw; t < T; t += nw) {
    int dst[kMaxTopk], pos[kMaxTopk];
#pragma unroll
    for (int k = 0; k < kMaxTopk; k++) {
      dst[k] = 0;
      pos[k] = -1;
      if (k < topk) {
        const int id = ids[t * topk + k];
        const int p = pairPos[t * topk + k];
        if (id >= 0 && id < numExperts && p >= 0) {
          const int d = id / epr;
          const int r = info->offs[d] + p;
          dst[k] = d;
          pos[k] = r < cap ? r : -1;
        }
      }
    }
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    for (int c0 = 0; c0 < H; c0 += 256 * kChunkUnroll) {
      uint4 raw[kChunkUnroll];
      loadChunks(xr, c0, H, lane, raw);
#pragma unroll
      for (int u = 0; u < kChunkUnroll; u++) {
        if (c0 + u * 256 >= H) break;  // warp-uniform
        const int col = c0 + u * 256 + lane * 8;
        const bool active = col < H;
        float f[8];
        unpackBf16x8(raw[u], f);
        float scale;
        const uint2 q = quantize8(f, active, &scale);
        if (active) {
#pragma unroll
          for (int k = 0; k < kMaxTopk; k++) {
            if (pos[k] < 0) continue;
            char* db = c.moe[dst[k]];
            *reinterpret_cast<uint2*>(db + L.rxData + static_cast<size_t>(pos[k]) * H + col) = q;
            if ((lane & 15) == 0)
              *reinterpret_cast<float*>(db + L.rxScale + (static_cast<size_t>(pos[k]) * nb + col / 128) * 4) =
                  scale;
          }
        }
      }
    }
    if (lane < topk) {
      int myPos = -1, myDst = 0;
#pragma unroll
      for (int k = 0; k < kMaxTopk; k++)
        if (k == lane) {
          myPos = pos[k];
          myDst = dst[k];
        }
      if (myPos >= 0) {
        const int id = ids[t * topk + lane];
        char* db = c.moe[myDst];
        *reinterpret_cast<int4*>(db + L.rxMeta + static_cast<size_t>(myPos) * 16) = make_int4(me, t, lane, id % epr);
        *reinterpret_cast<float*>(db + L.rxW + static_cast<size_t>(myPos) * 4) = w[t * topk + lane];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    dev::fenceSys();
    if (lastBlock(c, 0, e)) {
      dev::fenceSys();
      for (int q = 0; q < n; q++) redAddReleaseSys(ctrl32(c, q, dev::kMoeDispDoneOff) + me, 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// dispatch 3: wait for every source, dequantise into the caller's buffers
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) moeReceive(DevComm c, Layout L, __nv_bfloat16* recvX, int* recvMeta,
                                                       float* recvW, int H) {
  __shared__ uint32_t sE;
  __shared__ int sFail;
  const int n = c.nranks, me = c.rank;
  if (threadIdx.x == 0) {
    sE = *ctrl32(c, me, dev::kMoeDispEpochOff) + 1u;
    sFail = 0;
  }
  __syncthreads();
  const uint32_t e = sE;
  if (threadIdx.x < n &&
      !dev::waitAcquire(c, ctrl32(c, me, dev::kMoeDispDoneOff) + threadIdx.x, e, dev::kWhereMoe, 100 + threadIdx.x,
                        32))
    sFail = 1;
  __syncthreads();
  const char* base = c.moe[me];
  const Info* info = reinterpret_cast<const Info*>(base + L.info);
  const int recv = sFail ? 0 : info->recv;
  const int lane = threadIdx.x & 31;
  const int nb = H / 128;
  const int gw = blockIdx.x * (kThreads / 32) + threadIdx.x / 32, nw = gridDim.x * (kThreads / 32);
  for (int i = gw; i < recv; i += nw) {
    const char* row = base + L.rxData + static_cast<size_t>(i) * H;
    const float* sc = reinterpret_cast<const float*>(base + L.rxScale) + static_cast<size_t>(i) * nb;
    for (int c0 = 0; c0 < H; c0 += 256 * kChunkUnroll) {
      uint2 q[kChunkUnroll];
      float sv[kChunkUnroll];
#pragma unroll
      for (int u = 0; u < kChunkUnroll; u++) {
        const int col = c0 + u * 256 + lane * 8;
        if (col < H) {
          q[u] = __ldcg(reinterpret_cast<const uint2*>(row + col));
          sv[u] = __ldcg(sc + col / 128);
        }
      }
#pragma unroll
      for (int u = 0; u < kChunkUnroll; u++) {
        const int col = c0 + u * 256 + lane * 8;
        if (col < H) {
          float f[8];
          fromFp8x8(q[u], f);
#pragma unroll
          for (int j = 0; j < 8; j++) f[j] *= sv[u];
          *reinterpret_cast<uint4*>(recvX + static_cast<size_t>(i) * H + col) = packBf16x8(f);
        }
      }
    }
    if (lane == 0) {
      reinterpret_cast<int4*>(recvMeta)[i] = __ldcg(reinterpret_cast<const int4*>(base + L.rxMeta) + i);
      recvW[i] = __ldcg(reinterpret_cast<const float*>(base + L.rxW) + i);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && lastBlock(c, 1, e)) *ctrl32(c, me, dev::kMoeDispEpochOff) = e;
}

// ---------------------------------------------------------------------------
// combine 1: weighted expert rows back to their source slots
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) moeCombinePush(DevComm c, Layout L, const __nv_bfloat16* y,
                                                           const int* recvMeta, const float* recvW,
                                                           const int* recvCount, int H, int topk, int srcTokensCap) {
  __shared__ uint32_t sE;
  const int n = c.nranks, me = c.rank;
  if (threadIdx.x == 0) sE = *ctrl32(c, me, dev::kMoeCombEpochOff) + 1u;
  __syncthreads();
  const uint32_t e = sE;
  const int recv = *recvCount;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (kThreads / 32) + threadIdx.x / 32, nw = gridDim.x * (kThreads / 32);
  for (int i = gw; i < recv; i += nw) {
    const int4 meta = reinterpret_cast<const int4*>(recvMeta)[i];
    const float wt = recvW[i];
    const int slot = meta.y * topk + meta.z;
    if (meta.x < 0 || meta.x >= n || meta.z < 0 || meta.z >= topk || slot < 0 || slot >= srcTokensCap) continue;
    char* dst = c.moe[meta.x] + L.comb + static_cast<size_t>(slot) * H * 2;
    const uint4* yr = reinterpret_cast<const uint4*>(y + static_cast<size_t>(i) * H);
    for (int c0 = 0; c0 < H; c0 += 256 * kChunkUnroll) {
      uint4 raw[kChunkUnroll];
      loadChunks(yr, c0, H, lane, raw);
#pragma unroll
      for (int u = 0; u < kChunkUnroll; u++) {
        const int col = c0 + u * 256 + lane * 8;
        if (col < H) {
          float f[8];
          unpackBf16x8(raw[u], f);
#pragma unroll
          for (int j = 0; j < 8; j++) f[j] *= wt;
          *reinterpret_cast<uint4*>(dst + static_cast<size_t>(col) * 2) = packBf16x8(f);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    dev::fenceSys();
    if (lastBlock(c, 2, e)) {
      dev::fenceSys();
      for (int q = 0; q < n; q++) redAddReleaseSys(ctrl32(c, q, dev::kMoeCombDoneOff) + me, 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// combine 2: wait for every expert rank, sum the k slots of each token
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) moeCombineReduce(DevComm c, Layout L, __nv_bfloat16* out, int T, int H,
                                                             int topk) {
  __shared__ uint32_t sE;
  __shared__ int sFail;
  const int n = c.nranks, me = c.rank;
  if (threadIdx.x == 0) {
    sE = *ctrl32(c, me, dev::kMoeCombEpochOff) + 1u;
    sFail = 0;
  }
  __syncthreads();
  const uint32_t e = sE;
  if (threadIdx.x < n &&
      !dev::waitAcquire(c, ctrl32(c, me, dev::kMoeCombDoneOff) + threadIdx.x, e, dev::kWhereMoe, 200 + threadIdx.x,
                        32))
    sFail = 1;
  __syncthreads();
  const char* comb = c.moe[me] + L.comb;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (kThreads / 32) + threadIdx.x / 32, nw = gridDim.x * (kThreads / 32);
  for (int t = sFail ? T : gw; t < T; t += nw) {
    for (int c0 = 0; c0 < H; c0 += 256) {
      const int col = c0 + lane * 8;
      if (col >= H) continue;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < topk; k++) {
        float f[8];
        unpackBf16x8(__ldcg(reinterpret_cast<const uint4*>(comb + (static_cast<size_t>(t) * topk + k) * H * 2 +
                                                           static_cast<size_t>(col) * 2)),
                     f);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] += f[j];
      }
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + col) = packBf16x8(acc);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && lastBlock(c, 3, e)) *ctrl32(c, me, dev::kMoeCombEpochOff) = e;
}

// ---------------------------------------------------------------------------
// single rank: the same quantise / dequantise and weighted sum, locally
// ---------------------------------------------------------------------------
int localGrid() {
  static const int g = [] {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms * kLocalBlocksPerSm;
  }();
  return g;
}

__global__ void __launch_bounds__(kThreads) moeLocalDispatch(const __nv_bfloat16* x, const int* ids, const float* w,
                                                             int T, int H, int topk, int numExperts,
                                                             __nv_bfloat16* recvX, int* recvMeta, float* recvW,
                                                             int* recvCount) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (kThreads / 32) + threadIdx.x / 32, nw = gridDim.x * (kThreads / 32);
  const int P = T * topk;
  if (blockIdx.x == 0 && threadIdx.x == 0) *recvCount = P;
  for (int i = gw; i < P; i += nw) {
    const int t = i / topk;
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    for (int c0 = 0; c0 < H; c0 += 256 * kChunkUnroll) {
      uint4 raw[kChunkUnroll];
      loadChunks(xr, c0, H, lane, raw);
#pragma unroll
      for (int u = 0; u < kChunkUnroll; u++) {
        if (c0 + u * 256 >= H) break;  // warp-uniform
        const int col = c0 + u * 256 + lane * 8;
        const bool active = col < H;
        float f[8];
        unpackBf16x8(raw[u], f);
        float scale;
        const uint2 q = quantize8(f, active, &scale);
        if (active) {
          fromFp8x8(q, f);
#pragma unroll
          for (int j = 0; j < 8; j++) f[j] *= scale;
          *reinterpret_cast<uint4*>(recvX + static_cast<size_t>(i) * H + col) = packBf16x8(f);
        }
      }
    }
    if (lane == 0) {
      const int id = ids[i];
      reinterpret_cast<int4*>(recvMeta)[i] = make_int4(0, t, i - t * topk, id >= 0 && id < numExperts ? id : -1);
      recvW[i] = w[i];
    }
  }
}

__global__ void __launch_bounds__(kThreads) moeLocalCombine(const __nv_bfloat16* y, const float* recvW,
                                                            __nv_bfloat16* out, int T, int H, int topk) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (kThreads / 32) + threadIdx.x / 32, nw = gridDim.x * (kThreads / 32);
  for (int t = gw; t < T; t += nw) {
    for (int c0 = 0; c0 < H; c0 += 256) {
      const int col = c0 + lane * 8;
      if (col >= H) continue;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < topk; k++) {
        const int i = t * topk + k;
        const float wt = recvW[i];
        float f[8];
        unpackBf16x8(reinterpret_cast<const uint4*>(y + static_cast<size_t>(i) * H)[col / 8], f);
        // Same rounding as the multi-rank path: the weighted row is rounded to
        // bf16 before the sum.
        float r[8];
#pragma unroll
        for (int j = 0; j < 8; j++) r[j] = f[j] * wt;
        unpackBf16x8(packBf16x8(r), f);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] += f[j];
      }
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + col) = packBf16x8(acc);
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace moe
}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclMoeDispatchFp8(const void* x, const int* topkIds, const float* topkW, void* recvX,
                                           int* recvMeta, float* recvW, int* recvCount, int T, int H, int topk,
                                           int numExperts, int capacity, vcclComm_t comm, vcclStream_t stream) {
  TraceRange trace("vccl MoeDispatchFp8");
  if (comm == nullptr || !x || !topkIds || !topkW || !recvX || !recvMeta || !recvW || !recvCount) {
    return vcclInvalidArgument;
  }
  if (T < 0 || H <= 0 || H % 128 != 0 || topk < 1 || topk > moe::kMaxTopk || numExperts < 1 || capacity < 1 ||
      static_cast<long long>(T) * topk > capacity || !moe::aligned16(x) || !moe::aligned16(recvX) ||
      !moe::aligned16(recvMeta)) {
    VERR("vcclMoeDispatchFp8: need H %% 128 == 0, 1 <= topk <= %d, T * topk <= capacity and 16-byte aligned "
         "x / recvX / recvMeta (T=%d H=%d topk=%d capacity=%d)",
         moe::kMaxTopk, T, H, topk, capacity);
    return vcclInvalidArgument;
  }
  if (comm->aborted.load() || !comm->dev) return vcclInvalidUsage;
  const int n = comm->nranks;
  if (numExperts % n != 0) {
    VERR("vcclMoeDispatchFp8: %d experts do not split evenly over %d ranks", numExperts, n);
    return vcclInvalidArgument;
  }
  vcclResult_t st = comm->pollDeviceStatus();
  if (st != vcclSuccess) {
    comm->noteError(st);
    return vcclInvalidUsage;
  }
  cudaSetDevice(comm->dev->device);
  if (!devicePointers(comm->dev->device, {x, topkIds, topkW, recvX, recvMeta, recvW, recvCount}, "vcclMoeDispatchFp8"))
    return vcclInvalidArgument;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  OrderedLaunch ord(comm->dev.get(), s);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* rx = static_cast<__nv_bfloat16*>(recvX);
  if (n == 1) {
    moe::moeLocalDispatch<<<moe::localGrid(), moe::kThreads, 0, s>>>(xb, topkIds, topkW, T, H, topk, numExperts, rx,
                                                               recvMeta, recvW, recvCount);
    if (cudaGetLastError() != cudaSuccess) return vcclUnhandledError;
    comm->noteCall("moe dispatch (fp8)", "one rank: local", static_cast<size_t>(T) * H * 2);
    return vcclSuccess;
  }
  const moe::Layout L = moe::layoutFor(capacity, H);
  VTRY(deviceStateEnsureMoe(comm->dev.get(), comm->bootstrap.get(), L.total));
  const dev::DevComm& dc = comm->dev->dc;
  const int epr = numExperts / n;
  moe::moeCount<<<1, 1024, 0, s>>>(dc, topkIds, T * topk, epr, numExperts, capacity, L, recvCount);
  moe::moePush<<<moe::kGrid, moe::kThreads, 0, s>>>(dc, xb, topkIds, topkW, T, H, topk, epr, numExperts, capacity,
                                                    L);
  moe::moeReceive<<<moe::kGrid, moe::kThreads, 0, s>>>(dc, L, rx, recvMeta, recvW, H);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    VERR("vcclMoeDispatchFp8 launch: %s", cudaGetErrorString(e));
    return vcclUnhandledError;
  }
  comm->noteCall("moe dispatch (fp8)", "count, push, receive", static_cast<size_t>(T) * H * 2);
  return vcclSuccess;
}

extern "C" vcclResult_t vcclMoeCombine(const void* expertOut, const int* recvMeta, const float* recvW,
                                       const int* recvCount, void* out, int T, int H, int topk, int capacity,
                                       vcclComm_t comm, vcclStream_t stream) {
  TraceRange trace("vccl MoeCombine");
  if (comm == nullptr || !expertOut || !recvMeta || !recvW || !recvCount || !out) return vcclInvalidArgument;
  if (T < 0 || H <= 0 || H % 128 != 0 || topk < 1 || topk > moe::kMaxTopk || capacity < 1 ||
      static_cast<long long>(T) * topk > capacity || !moe::aligned16(expertOut) || !moe::aligned16(out) ||
      !moe::aligned16(recvMeta)) {
    VERR("vcclMoeCombine: need H %% 128 == 0, 1 <= topk <= %d, T * topk <= capacity and 16-byte aligned buffers",
         moe::kMaxTopk);
    return vcclInvalidArgument;
  }
  if (comm->aborted.load() || !comm->dev) return vcclInvalidUsage;
  vcclResult_t st = comm->pollDeviceStatus();
  if (st != vcclSuccess) {
    comm->noteError(st);
    return vcclInvalidUsage;
  }
  cudaSetDevice(comm->dev->device);
  if (!devicePointers(comm->dev->device, {expertOut, recvMeta, recvW, recvCount, out}, "vcclMoeCombine"))
    return vcclInvalidArgument;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  OrderedLaunch ord(comm->dev.get(), s);
  const auto* y = static_cast<const __nv_bfloat16*>(expertOut);
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (comm->nranks == 1) {
    moe::moeLocalCombine<<<moe::localGrid(), moe::kThreads, 0, s>>>(y, recvW, o, T, H, topk);
    if (cudaGetLastError() != cudaSuccess) return vcclUnhandledError;
    comm->noteCall("moe combine", "one rank: local", static_cast<size_t>(T) * H * 2);
    return vcclSuccess;
  }
  const moe::Layout L = moe::layoutFor(capacity, H);
  if (comm->dev->dc.moeBytes < L.total) {
    VERR("vcclMoeCombine: no dispatch with this capacity and hidden size ran on this communicator");
    return vcclInvalidUsage;
  }
  const dev::DevComm& dc = comm->dev->dc;
  moe::moeCombinePush<<<moe::kGrid, moe::kThreads, 0, s>>>(dc, L, y, recvMeta, recvW, recvCount, H, topk, capacity);
  moe::moeCombineReduce<<<moe::kGrid, moe::kThreads, 0, s>>>(dc, L, o, T, H, topk);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    VERR("vcclMoeCombine launch: %s", cudaGetErrorString(e));
    return vcclUnhandledError;
  }
  comm->noteCall("moe combine", "push, reduce", static_cast<size_t>(T) * H * 2);
  return vcclSuccess;
}
