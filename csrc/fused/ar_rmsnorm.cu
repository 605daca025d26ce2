// SPDX-License-Identifier: Apache-2.0
// All-reduce fused with residual add and RMSNorm (bf16).
//
//   x        = residual + sum_over_ranks(partial)      (fp32 math)
//   residual = bf16(x)                                  (in place, every rank)
//   out      = bf16(x * rsqrt(mean(x^2) + eps) * weight)
//
// This is the decode-time tail of every attention-out and MLP-out
// projection in a tensor-parallel transformer; the reference's vLLM
// communicator does it as an all_reduce followed by separate torch ops
// (reference: python/vccl/torch_comm.py:132-139, python/tests/
// test_e2e_tp.py:80-81).  Two kernels:
//
//  * LL (small batches): every rank writes its partial as LL lines into
//    every peer (one NVLink hop, no barrier).  Rows are normalised by 8-CTA
//    thread-block clusters: each CTA owns 1/8 of a row and the row's sum of
//    squares is combined through distributed shared memory.
//  * Two-shot (large batches): rows are split among ranks; partial rows are
//    pushed to their owner, the owner adds, normalises and publishes x and
//    out, and every rank pulls the rows it does not own.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common/log.h"
#include "common/trace.h"
#include "kernels/collectives.cuh"
#include "runtime/comm.h"
#include "vccl_tp.h"

namespace cg = cooperative_groups;

namespace vccl {
namespace dev {

constexpr int kNormThreads = 512;
constexpr int kClusterCtas = 8;

__device__ __forceinline__ void bf16x4ToFloat(uint64_t w, float (&f)[4]) {
  const uint32_t lo = static_cast<uint32_t>(w), hi = static_cast<uint32_t>(w >> 32);
  f[0] = __uint_as_float(lo << 16);
  f[1] = __uint_as_float(lo & 0xffff0000u);
  f[2] = __uint_as_float(hi << 16);
  f[3] = __uint_as_float(hi & 0xffff0000u);
}
__device__ __forceinline__ uint64_t floatToBf16x4(const float (&f)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
  return static_cast<uint64_t>(*reinterpret_cast<uint32_t*>(&a)) |
         (static_cast<uint64_t>(*reinterpret_cast<uint32_t*>(&b)) << 32);
}

__device__ __forceinline__ float blockSum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < blockDim.x / 32) t = scratch[threadIdx.x];
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) scratch[32] = t;
  }
  __syncthreads();
  return scratch[32];
}

struct NormArgs {
  const char* partial;
  char* residual;
  const char* weight;
  char* out;
  int rows;
  int hidden;
  float eps;
};

// LL variant.  Grid = the communicator's llBlocks CTAs in clusters of 8; every CTA bumps its LL
// epoch once.  rows*hidden*2 <= kLLMaxBytes, hidden % (4*8) == 0.
constexpr int kMaxWordsPerThread = 4;

__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kNormThreads)
    arRmsNormLL(DevComm c, NormArgs a) {
  const uint32_t e = llEpoch(c);
  const uint32_t par = e & 1u;
  const int n = c.nranks, me = c.rank;
  const size_t bytes = static_cast<size_t>(a.rows) * a.hidden * 2;
  const size_t words = bytes / 8;
  // 1. push my partial to every peer (any CTA may push any word).
  {
    size_t w0, w1;
    blockRange(words, gridDim.x, blockIdx.x, 1, &w0, &w1);
    for (size_t w = w0 + threadIdx.x; w < w1; w += blockDim.x) {
      const uint64_t word = *reinterpret_cast<const uint64_t*>(a.partial + w * 8);
      for (int k = 1; k < n; k++) llPut(c, (me + k) % n, par, e, w, word);
    }
  }
  // 2. rows: cluster `cl` handles rows cl, cl + clusters, ...
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float scratch[33];
  __shared__ float clusterPartial;
  const int cl = blockIdx.x / kClusterCtas;
  const int clusters = gridDim.x / kClusterCtas;
  const int part = static_cast<int>(cluster.block_rank());
  const int wpr = a.hidden / 4;  // 8-byte words per row
  const int wPerCta = wpr / kClusterCtas;
  const float invH = 1.0f / static_cast<float>(a.hidden);
  bool ok = true;
  for (int row = cl; row < a.rows; row += clusters) {
    float x[kMaxWordsPerThread][4];
    float ss = 0.f;
    int cnt = 0;
    for (int i = threadIdx.x; i < wPerCta && ok; i += blockDim.x, cnt++) {
      const size_t w = static_cast<size_t>(row) * wpr + part * wPerCta + i;
      float acc[4], t[4];
      bf16x4ToFloat(*reinterpret_cast<const uint64_t*>(a.partial + w * 8), acc);
      for (int k = 1; k < n && ok; k++) {
        uint64_t v;
        ok = llWait(c, llSlot(c, me, par, (me + k) % n) + w * 16, e, &v);
        bf16x4ToFloat(v, t);
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] += t[j];
      }
      bf16x4ToFloat(*reinterpret_cast<const uint64_t*>(a.residual + w * 8), t);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        x[cnt][j] = acc[j] + t[j];
        ss += x[cnt][j] * x[cnt][j];
      }
    }
    // Every CTA of the cluster must reach the cluster barriers, even after a
    // failed wait, so failure is only acted on after the row.
    const float blockSs = blockSum(ss, scratch);
    if (threadIdx.x == 0) clusterPartial = blockSs;
    cluster.sync();
    float total = 0.f;
    if (threadIdx.x < kClusterCtas) total = *cluster.map_shared_rank(&clusterPartial, threadIdx.x);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    total = __shfl_sync(0xffffffffu, total, 0);
    if (threadIdx.x < 32) scratch[32] = total;
    cluster.sync();
    __syncthreads();
    const float rstd = rsqrtf(scratch[32] * invH + a.eps);
    cnt = 0;
    for (int i = threadIdx.x; i < wPerCta && ok; i += blockDim.x, cnt++) {
      const size_t w = static_cast<size_t>(row) * wpr + part * wPerCta + i;
      float wt[4], o[4];
      bf16x4ToFloat(*reinterpret_cast<const uint64_t*>(a.weight + (w % wpr) * 8), wt);
#pragma unroll
      for (int j = 0; j < 4; j++) o[j] = x[cnt][j] * rstd * wt[j];
      *reinterpret_cast<uint64_t*>(a.residual + w * 8) = floatToBf16x4(x[cnt]);
      *reinterpret_cast<uint64_t*>(a.out + w * 8) = floatToBf16x4(o);
    }
    __syncthreads();
  }
}

// Two-shot variant.  Rank q owns rows [q*R/n, (q+1)*R/n).  Block b handles
// local rows b, b+G, ... of every chunk in every phase, so each phase only
// depends on block b of the other ranks.
__device__ __forceinline__ int rowBegin(int q, int rows, int n) {
  return static_cast<int>((static_cast<long long>(rows) * q) / n);
}

constexpr int kMaxPacksPerThread = 8;  // hidden <= 512 threads * 8 packs * 8 = 32768

// Copies `count` rows of rowBytes (a multiple of 16) with the whole block,
// row i from srcRow(i) to dstRow(i), keeping kCopyDepth 16-byte loads in
// flight per thread across rows: the pushes and pulls of a block's rows to
// and from its peers are latency-bound over NVLink when done row by row.
constexpr int kCopyDepth = 8;
template <typename Dst, typename Src>
__device__ __forceinline__ void copyRows(int count, size_t rowBytes, Dst&& dstRow, Src&& srcRow) {
  const size_t per = rowBytes / 16;
  const size_t total = per * static_cast<size_t>(count);
  const size_t nthr = blockDim.x;
  for (size_t base = threadIdx.x; base < total; base += nthr * kCopyDepth) {
    uint4 v[kCopyDepth];
#pragma unroll
    for (int u = 0; u < kCopyDepth; u++) {
      const size_t i = base + u * nthr;
      if (i < total) v[u] = ldCG(srcRow(static_cast<int>(i / per)) + (i % per) * 16);
    }
#pragma unroll
    for (int u = 0; u < kCopyDepth; u++) {
      const size_t i = base + u * nthr;
      if (i < total) stG(dstRow(static_cast<int>(i / per)) + (i % per) * 16, v[u]);
    }
  }
}

__global__ void __launch_bounds__(kNormThreads) arRmsNormTwoShot(DevComm c, NormArgs a, size_t slotRows) {
  const int blk = blockIdx.x, G = gridDim.x, n = c.nranks, me = c.rank;
  const size_t rowBytes = static_cast<size_t>(a.hidden) * 2;
  const size_t slotBytes = slotRows * rowBytes;
  char* mine = c.data[me];
  __shared__ float scratch[33];
  if (!blockBarrier(c, blk, kWhereStart)) return;
  // 1. push partial rows to their owners: this block's rows of every owner,
  //    all in flight together (row j: owner q = me + 1 + j / perOwner, local
  //    row blk + (j % perOwner) G of that owner's chunk)
  const int perOwner = (a.rows / n + 1 + G - 1) / G;  // upper bound of this block's rows per owner
  {
    auto owner = [&](int j) { return (me + 1 + j / perOwner) % n; };
    auto localRow = [&](int j) { return blk + (j % perOwner) * G; };
    auto valid = [&](int j) {
      const int q = owner(j);
      return rowBegin(q, a.rows, n) + localRow(j) < rowBegin(q + 1, a.rows, n);
    };
    // Compact the valid (owner, row) pairs into a small table so the copy
    // loop indexes rows directly.
    __shared__ int sRow[kMaxRanks * 64];
    __shared__ int sCount;
    if (threadIdx.x == 0) {
      int k = 0;
      for (int j = 0; j < (n - 1) * perOwner && k < kMaxRanks * 64; j++)
        if (valid(j)) sRow[k++] = j;
      sCount = k;
    }
    __syncthreads();
    const int total = sCount;
    const bool fits = (n - 1) * perOwner <= kMaxRanks * 64;
    if (fits) {
      copyRows(
          total, rowBytes,
          [&](int i) { return c.data[owner(sRow[i])] + me * slotBytes + localRow(sRow[i]) * rowBytes; },
          [&](int i) {
            const int q = owner(sRow[i]);
            return a.partial + (rowBegin(q, a.rows, n) + localRow(sRow[i])) * rowBytes;
          });
    } else {
      for (int q = 0; q < n; q++) {
        if (q == me) continue;
        const int r0 = rowBegin(q, a.rows, n), r1 = rowBegin(q + 1, a.rows, n);
        for (int lr = blk; r0 + lr < r1; lr += G)
          copyAny(c.data[q] + me * slotBytes + lr * rowBytes, a.partial + (r0 + lr) * rowBytes, rowBytes);
      }
    }
    __syncthreads();
  }
  if (!blockBarrier(c, blk, kWherePush)) return;
  // 2. reduce + residual + norm for my rows; publish x and out
  const int packs = a.hidden / 8;
  const float invH = 1.0f / static_cast<float>(a.hidden);
  {
    const int r0 = rowBegin(me, a.rows, n), r1 = rowBegin(me + 1, a.rows, n);
    for (int lr = blk; r0 + lr < r1; lr += G) {
      const size_t grow = static_cast<size_t>(r0 + lr) * rowBytes;
      float x[kMaxPacksPerThread][8];
      float ss = 0.f;
      int cnt = 0;
      for (int p = threadIdx.x; p < packs; p += blockDim.x, cnt++) {
        Pack<__nv_bfloat16> acc, res;
        acc.load(ldCG(a.partial + grow + p * 16));
        for (int k = 1; k < n; k++) {
          const int src = (me + k) % n;
          acc.fold<kSum>(ldCG(mine + src * slotBytes + lr * rowBytes + p * 16));
        }
        res.load(ldCG(a.residual + grow + p * 16));
#pragma unroll
        for (int j = 0; j < 8; j++) {
          x[cnt][j] = acc.v[j] + res.v[j];
          ss += x[cnt][j] * x[cnt][j];
        }
      }
      const float rstd = rsqrtf(blockSum(ss, scratch) * invH + a.eps);
      cnt = 0;
      for (int p = threadIdx.x; p < packs; p += blockDim.x, cnt++) {
        Pack<__nv_bfloat16> xo, oo, wt;
        wt.load(ldCG(a.weight + p * 16));
#pragma unroll
        for (int j = 0; j < 8; j++) {
          xo.v[j] = x[cnt][j];
          oo.v[j] = x[cnt][j] * rstd * wt.v[j];
        }
        const uint4 xr = xo.pack(), orw = oo.pack();
        stG(a.residual + grow + p * 16, xr);
        stG(a.out + grow + p * 16, orw);
        stG(mine + n * slotBytes + lr * rowBytes + p * 16, xr);
        stG(mine + (n + 1) * slotBytes + lr * rowBytes + p * 16, orw);
      }
    }
  }
  if (!blockBarrier(c, blk, kWhereReduce)) return;
  // 3. pull the rows owned by the other ranks (residual and output of each),
  //    all of this block's rows in flight together
  {
    __shared__ int sPull[2 * kMaxRanks * 64];
    __shared__ int sPullCount;
    const bool fits = 2 * (n - 1) * perOwner <= 2 * kMaxRanks * 64;
    if (threadIdx.x == 0) {
      int k = 0;
      for (int j = 0; fits && j < (n - 1) * perOwner; j++) {
        const int q = (me + 1 + j / perOwner) % n;
        const int lr = blk + (j % perOwner) * G;
        if (rowBegin(q, a.rows, n) + lr < rowBegin(q + 1, a.rows, n)) {
          sPull[k++] = 2 * j;      // residual row
          sPull[k++] = 2 * j + 1;  // output row
        }
      }
      sPullCount = k;
    }
    __syncthreads();
    auto ownerOf = [&](int e) { return (me + 1 + (e / 2) / perOwner) % n; };
    auto lrOf = [&](int e) { return blk + ((e / 2) % perOwner) * G; };
    if (fits) {
      copyRows(
          sPullCount, rowBytes,
          [&](int i) {
            const int e = sPull[i];
            const int q = ownerOf(e);
            return (e & 1 ? a.out : a.residual) + (rowBegin(q, a.rows, n) + lrOf(e)) * rowBytes;
          },
          [&](int i) {
            const int e = sPull[i];
            return c.data[ownerOf(e)] + ((e & 1) ? n + 1 : n) * slotBytes + lrOf(e) * rowBytes;
          });
    } else {
      for (int q = 0; q < n; q++) {
        if (q == me) continue;
        const int r0 = rowBegin(q, a.rows, n), r1 = rowBegin(q + 1, a.rows, n);
        for (int lr = blk; r0 + lr < r1; lr += G) {
          copyAny(a.residual + (r0 + lr) * rowBytes, c.data[q] + n * slotBytes + lr * rowBytes, rowBytes);
          copyAny(a.out + (r0 + lr) * rowBytes, c.data[q] + (n + 1) * slotBytes + lr * rowBytes, rowBytes);
        }
      }
    }
  }
}

// Single rank: residual += partial; out = norm(residual) * weight.
__global__ void __launch_bounds__(kNormThreads) addRmsNormLocal(NormArgs a) {
  __shared__ float scratch[33];
  const size_t rowBytes = static_cast<size_t>(a.hidden) * 2;
  const int packs = a.hidden / 8;
  const float invH = 1.0f / static_cast<float>(a.hidden);
  for (int row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const size_t g = row * rowBytes;
    float x[kMaxPacksPerThread][8];
    float ss = 0.f;
    int cnt = 0;
    for (int p = threadIdx.x; p < packs; p += blockDim.x, cnt++) {
      Pack<__nv_bfloat16> pa, re;
      pa.load(ldCG(a.partial + g + p * 16));
      re.load(ldCG(a.residual + g + p * 16));
#pragma unroll
      for (int j = 0; j < 8; j++) {
        x[cnt][j] = pa.v[j] + re.v[j];
        ss += x[cnt][j] * x[cnt][j];
      }
    }
    const float rstd = rsqrtf(blockSum(ss, scratch) * invH + a.eps);
    cnt = 0;
    for (int p = threadIdx.x; p < packs; p += blockDim.x, cnt++) {
      Pack<__nv_bfloat16> xo, oo, wt;
      wt.load(ldCG(a.weight + p * 16));
#pragma unroll
      for (int j = 0; j < 8; j++) {
        xo.v[j] = x[cnt][j];
        oo.v[j] = x[cnt][j] * rstd * wt.v[j];
      }
      stG(a.residual + g + p * 16, xo.pack());
      stG(a.out + g + p * 16, oo.pack());
    }
    __syncthreads();
  }
}

}  // namespace dev
}  // namespace vccl

using namespace vccl;

extern "C" vcclResult_t vcclAllReduceAddRMSNorm(const void* partial, void* residual, const void* weight, void* out,
                                                size_t rows, size_t hidden, float eps, vcclDataType_t datatype,
                                                vcclComm_t comm, vcclStream_t stream) {
  TraceRange trace("vccl AllReduceAddRMSNorm");
  if (comm == nullptr || partial == nullptr || residual == nullptr || weight == nullptr || out == nullptr)
    return vcclInvalidArgument;
  if (datatype != vcclBfloat16 || hidden % 32 != 0 || hidden > 32768 || rows == 0) {
    VERR("vcclAllReduceAddRMSNorm: bf16, hidden %% 32 == 0 and hidden <= 32768 required");
    return vcclInvalidArgument;
  }
  if (((reinterpret_cast<uintptr_t>(partial) | reinterpret_cast<uintptr_t>(residual) |
        reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
    return vcclInvalidArgument;
  if (comm->aborted.load() || !comm->dev) return vcclInvalidUsage;
  vcclResult_t st = comm->pollDeviceStatus();
  if (st != vcclSuccess) {
    comm->noteError(st);
    return vcclInvalidUsage;
  }
  cudaSetDevice(comm->dev->device);
  if (!devicePointers(comm->dev->device, {partial, residual, weight, out}, "vcclAllReduceAddRMSNorm")) return vcclInvalidArgument;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  OrderedLaunch ord(comm->dev.get(), s);
  dev::NormArgs a{static_cast<const char*>(partial), static_cast<char*>(residual), static_cast<const char*>(weight),
                  static_cast<char*>(out), static_cast<int>(rows), static_cast<int>(hidden), eps};
  const int n = comm->nranks;
  const size_t bytes = rows * hidden * 2;
  const char* path = "two-shot";
  if (n == 1) {
    const int grid = static_cast<int>(rows < 1024 ? rows : 1024);
    dev::addRmsNormLocal<<<grid, dev::kNormThreads, 0, s>>>(a);
    path = "one rank: add + RMSNorm";
  } else if (bytes <= comm->dev->llMaxBytes * 4 && bytes <= dev::kLLMaxBytes &&
             hidden / 4 / dev::kClusterCtas <= dev::kNormThreads * dev::kMaxWordsPerThread) {
    dev::arRmsNormLL<<<comm->dev->llBlocks, dev::kNormThreads, 0, s>>>(comm->dev->dc, a);
    path = "LL, 8-CTA clusters";
  } else {
    const size_t maxRows = (rows + n - 1) / n;
    const size_t slotRows = comm->dev->dc.dataBytes / (n + 2) / (hidden * 2);
    if (maxRows > slotRows) {
      VERR("vcclAllReduceAddRMSNorm: %zu rows exceed the staging capacity (%zu per rank)", rows, slotRows * n);
      return vcclInvalidArgument;
    }
    int grid = static_cast<int>(maxRows < static_cast<size_t>(comm->dev->nblocks) ? maxRows : comm->dev->nblocks);
    dev::arRmsNormTwoShot<<<grid, dev::kNormThreads, 0, s>>>(comm->dev->dc, a, slotRows);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    VERR("vcclAllReduceAddRMSNorm launch: %s", cudaGetErrorString(e));
    return vcclUnhandledError;
  }
  comm->noteCall("all-reduce + residual + RMSNorm", path, bytes);
  return vcclSuccess;
}
