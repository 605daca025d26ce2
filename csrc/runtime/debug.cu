// SPDX-License-Identifier: Apache-2.0
// Diagnostics: cross-GPU barrier latency microbenchmark.
//
// vcclxBarrierBench runs `iters` back-to-back block barriers in one kernel
// (every rank must call it with the same arguments) and returns the
// per-barrier time in microseconds.  Variants compare the signalling /
// polling memory orders so the collective kernels can use the cheapest
// correct one.  Waits are bounded like every other wait in the library.
#include <cuda_runtime.h>

#include "common/env.h"
#include "kernels/collectives.cuh"
#include "runtime/comm.h"
#include "vccl_x.h"

namespace vccl {
namespace dev {

__device__ __forceinline__ uint32_t ldAcquireSys32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
template <int V>
__device__ __forceinline__ bool benchBarrier(const DevComm& c, uint32_t e) {
  const int t = threadIdx.x;
  bool ok = true;
  __syncthreads();
  if (t < c.nranks) {
    uint32_t* remote = ctrlAt<uint32_t>(c, t, kBarFlagsOff) + blockIdx.x * kMaxRanks + c.rank;
    const uint32_t* mine = ctrlAt<uint32_t>(c, c.rank, kBarFlagsOff) + blockIdx.x * kMaxRanks + t;
    if (V == 0) {  // fence + relaxed store; relaxed poll + fence
      fenceSys();
      stRelaxedSys(remote, e);
      ok = waitAtLeast(c, mine, e, kWhereStart, t);
    } else if (V == 1) {  // release store; acquire poll
      stReleaseSys32(remote, e);
      const uint64_t t0 = globalTimerNs();
      while (static_cast<int32_t>(ldAcquireSys32(mine) - e) < 0) {
        if (globalTimerNs() - t0 > c.timeoutNs) return false;
      }
    } else if (V == 2) {  // volatile store / poll, no fences (timing floor only)
      *reinterpret_cast<volatile uint32_t*>(remote) = e;
      const uint64_t t0 = globalTimerNs();
      while (static_cast<int32_t>(*reinterpret_cast<const volatile uint32_t*>(mine) - e) < 0) {
        if (globalTimerNs() - t0 > c.timeoutNs) return false;
      }
    } else {  // release store; relaxed poll + acquire fence
      stReleaseSys32(remote, e);
      const uint64_t t0 = globalTimerNs();
      while (static_cast<int32_t>(ldRelaxedSys(mine) - e) < 0) {
        if (globalTimerNs() - t0 > c.timeoutNs) return false;
      }
      fenceSys();
    }
  }
  __syncthreads();
  return ok;
}

template <int V>
__global__ void barrierBenchKernel(DevComm c, int iters) {
  __shared__ uint32_t base;
  if (threadIdx.x == 0) base = ctrlAt<uint32_t>(c, c.rank, kBarEpochOff)[blockIdx.x];
  __syncthreads();
  for (int i = 1; i <= iters; i++)
    if (!benchBarrier<V>(c, base + i)) break;
  if (threadIdx.x == 0) ctrlAt<uint32_t>(c, c.rank, kBarEpochOff)[blockIdx.x] = base + iters;
}

}  // namespace dev
}  // namespace vccl

extern "C" vcclResult_t vcclxBarrierBench(vcclComm_t comm, int iters, int nblocks, int variant, float* usPerBarrier) {
  if (comm == nullptr || !comm->dev || comm->nranks < 2 || nblocks < 1 || nblocks > vccl::dev::kMaxBlocks)
    return vcclInvalidArgument;
  cudaSetDevice(comm->dev->device);
  cudaStream_t s = comm->dev->stream;
  const vccl::dev::DevComm& dc = comm->dev->dc;
  vccl::OrderedLaunch ord(comm->dev.get(), s);  // after the communicator's earlier kernels
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, s);
  switch (variant) {
    case 0: vccl::dev::barrierBenchKernel<0><<<nblocks, 128, 0, s>>>(dc, iters); break;
    case 1: vccl::dev::barrierBenchKernel<1><<<nblocks, 128, 0, s>>>(dc, iters); break;
    case 2: vccl::dev::barrierBenchKernel<2><<<nblocks, 128, 0, s>>>(dc, iters); break;
    default: vccl::dev::barrierBenchKernel<3><<<nblocks, 128, 0, s>>>(dc, iters); break;
  }
  cudaEventRecord(b, s);
  cudaEventSynchronize(b);
  float ms = 0;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  *usPerBarrier = ms * 1000.0f / iters;
  return comm->pollDeviceStatus();
}

// Copy the optional fused-kernel event trace (VCCL_FUSED_TRACE=1 at
// communicator creation): *ctas rows of kFusedTraceSlots %globaltimer
// values (ns) per CTA, slots 0-18 from the last all-gather + GEMM (see
// AgHooks::trace) and 20-27 from the last GEMM + reduce-scatter (see
// fused/gemm_rs.cu).  Synchronises the device.
extern "C" vcclResult_t vcclxFusedTrace(vcclComm_t comm, unsigned long long* out, int* ctas) {
  if (comm == nullptr || out == nullptr || ctas == nullptr || !comm->dev) return vcclInvalidArgument;
  if (comm->dev->fusedTrace == nullptr) return vcclInvalidUsage;
  cudaSetDevice(comm->dev->device);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, comm->dev->device);
  if (sms > vccl::dev::kMaxFusedCtas) sms = vccl::dev::kMaxFusedCtas;
  if (cudaMemcpy(out, comm->dev->fusedTrace, static_cast<size_t>(sms) * vccl::dev::kFusedTraceSlots * 8,
                 cudaMemcpyDeviceToHost) != cudaSuccess)
    return vcclUnhandledError;
  *ctas = sms;
  return vcclSuccess;
}

namespace {
__global__ void guardScan(const unsigned char* p, size_t n, unsigned long long* bad) {
  unsigned long long mine = 0;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    mine += p[i] != vccl::dev::kGuardByte;
  if (mine) atomicAdd(bad, mine);
}
}  // namespace

// Debug layout check (VCCL_GUARDS=1 at communicator creation): counts the
// bytes of this rank's guard regions (past the ctrl, data and fused-op
// regions the kernels use) that no longer hold the fill pattern, i.e. bytes
// some kernel wrote out of bounds.  Synchronises the device.
// vcclInvalidUsage when the communicator has no guards.
extern "C" vcclResult_t vcclxCheckGuards(vcclComm_t comm, unsigned long long* badBytes) {
  if (comm == nullptr || badBytes == nullptr) return vcclInvalidArgument;
  if (!comm->dev || vccl::envLong("VCCL_GUARDS", 0) == 0) return vcclInvalidUsage;
  vccl::DeviceState* ds = comm->dev.get();
  cudaSetDevice(ds->device);
  unsigned long long* d = nullptr;
  if (cudaMalloc(&d, sizeof(*d)) != cudaSuccess) return vcclSystemError;
  cudaMemset(d, 0, sizeof(*d));
  const int me = comm->rank;
  bool any = false;
  for (const vccl::SymmetricBuffer* b : {&ds->ctrl, &ds->data, &ds->fused}) {
    if (b->va.empty() || b->bytes <= b->usable) continue;
    const unsigned char* p = reinterpret_cast<const unsigned char*>(b->va[me]) + b->usable;
    guardScan<<<64, 256>>>(p, b->bytes - b->usable, d);
    any = true;
  }
  cudaError_t e = cudaDeviceSynchronize();
  unsigned long long h = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return vcclUnhandledError;
  *badBytes = h;
  return any ? vcclSuccess : vcclInvalidUsage;
}
