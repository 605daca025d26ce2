// SPDX-License-Identifier: Apache-2.0
// Device-side building blocks shared by every collective kernel.
//
// Each rank owns two symmetric allocations that every peer maps:
//   ctrl: barrier flags, epochs, point-to-point counters, the LL region and
//         the point-to-point slot rings;
//   data: the staging region used by the barrier-based algorithms; when the
//         node supports NVLS it is also bound to a multicast object, and
//         `mcData` is its multicast address.
// All cross-GPU waits are bounded by %globaltimer.  A wait that runs out (or
// sees the host-mapped abort word) records an error in the host-mapped status
// words and makes its block return; it never traps.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vccl {
namespace dev {

constexpr int kMaxRanks = 8;     // one NVSwitch domain of an HGX B200 board
constexpr int kMaxBlocks = 128;  // largest grid of a barrier-based kernel
constexpr int kLLBlocks = 64;    // default grid of the LL kernels (VCCL_LL_BLOCKS, <= kMaxLLBlocks)
constexpr int kMaxLLBlocks = 256;
constexpr int kMaxChannels = 8;  // point-to-point channels per peer
constexpr int kP2pSlots = 4;     // ring depth of one channel

// ---- ctrl allocation layout (byte offsets) ---------------------------------
constexpr size_t kBarFlagsOff = 0;                                    // u32[kMaxBlocks][kMaxRanks], written by peers
constexpr size_t kBarEpochOff = kBarFlagsOff + kMaxBlocks * kMaxRanks * 4;  // u32[kMaxBlocks], local
constexpr size_t kLLEpochOff = kBarEpochOff + kMaxBlocks * 4;         // u32[kMaxLLBlocks], local
constexpr size_t kP2pHeadOff = 8192;                                  // u64[kMaxRanks][kMaxChannels], written by senders
constexpr size_t kP2pTailOff = kP2pHeadOff + kMaxRanks * kMaxChannels * 8;  // written by receivers
constexpr size_t kP2pSentOff = kP2pTailOff + kMaxRanks * kMaxChannels * 8;  // local
constexpr size_t kP2pRecvdOff = kP2pSentOff + kMaxRanks * kMaxChannels * 8; // local
constexpr size_t kMoeCountsOff = 32768;                               // u32[2][kMaxRanks][64], written by peers
// Fused GEMM + reduce-scatter / all-gather + GEMM counters (monotonic).
constexpr int kMaxFusedCtas = 256;
constexpr int kFusedTraceSlots = 32;  // event times per CTA in the optional AG+GEMM trace
constexpr int kFusedReduceBlocks = 64;
constexpr size_t kRsDoneOff = 65536;                        // u32[kMaxRanks]: peers' GEMM CTAs finished pushing
constexpr size_t kRsFreeOff = kRsDoneOff + 64;              // u32[kMaxRanks]: peers finished reducing my pushes
constexpr size_t kRsGemmCallsOff = kRsDoneOff + 256;        // u32[kMaxFusedCtas], local
constexpr size_t kRsReduceCallsOff = kRsGemmCallsOff + 1024; // u32[kFusedReduceBlocks], local
constexpr size_t kAgReadyOff = 69632;                       // u32[kMaxRanks]: peer staged its shard
constexpr size_t kAgTakenOff = kAgReadyOff + 64;            // u32[kMaxRanks]: peer finished pulling my shard
constexpr size_t kAgCallsOff = kAgReadyOff + 256;           // u32[kMaxFusedCtas], local
constexpr size_t kAgLocalReadyOff = kAgCallsOff + 1024;     // u32[kMaxRanks], local: shard copied into full X
constexpr size_t kAgStagedOff = kAgLocalReadyOff + 64;      // u32, local: CTAs that staged their slice
constexpr size_t kRsLocalDoneOff = kRsReduceCallsOff + 256; // u32, local: GEMM CTAs done pushing
constexpr size_t kRsLocalFreeOff = kRsLocalDoneOff + 4;     // u32, local: reduce blocks done
constexpr size_t kMoeOff = 73728;                           // MoE dispatch/combine counters
constexpr size_t kMoeDispDoneOff = kMoeOff;                 // u32[kMaxRanks], written by peers
constexpr size_t kMoeCombDoneOff = kMoeOff + 64;            // u32[kMaxRanks], written by peers
constexpr size_t kMoeDispEpochOff = kMoeOff + 128;          // u32, local: dispatch calls finished
constexpr size_t kMoeCombEpochOff = kMoeOff + 132;          // u32, local: combine calls finished
constexpr size_t kMoeBlocksOff = kMoeOff + 192;             // u32[4], local: per-kernel block counters
constexpr size_t kWinDescOff = 81920;                       // WinDesc[kMaxBlocks], read by peers (window calls)
constexpr size_t kWinA2aOff = 90112;                        // u64[kMaxBlocks][kMaxRanks][2]: all-to-all(v) receive table
// GEMM + reduce-scatter on CTA pairs (one kernel, reduction in the owner's epilogue)
constexpr int kRsMaxHalves = 8192;                          // 128-row x 256-column tiles of one owner's rows
constexpr size_t kRsArriveOff = 131072;                     // u32[kRsMaxHalves], written by peers: pushes landed
constexpr size_t kRsConsumedOff = kRsArriveOff + kRsMaxHalves * 4;   // u32[kRsMaxHalves], local: arrivals used
constexpr size_t kRsPairFreeOff = kRsConsumedOff + kRsMaxHalves * 4;  // u32, local: CTAs done this call
constexpr size_t kCtrlHeader = 1 << 20;
// The header's ranges must not overlap.
static_assert(kLLEpochOff + kMaxLLBlocks * 4 <= kP2pHeadOff, "epochs overlap the p2p counters");
static_assert(kP2pRecvdOff + kMaxRanks * kMaxChannels * 8 <= kMoeCountsOff, "p2p counters overlap the MoE rows");
static_assert(kMoeCountsOff + 2 * kMaxRanks * 64 * 4 <= kRsDoneOff, "MoE rows overlap the fused counters");
static_assert(kRsLocalFreeOff + 4 <= kAgReadyOff, "reduce-scatter counters overlap the all-gather counters");
static_assert(kAgStagedOff + 4 <= kMoeOff, "all-gather counters overlap the MoE counters");
static_assert(kMoeBlocksOff + 16 <= kWinDescOff, "MoE counters overlap the window descriptors");
static_assert(kWinDescOff + kMaxBlocks * 32 <= kWinA2aOff, "window descriptors overlap the all-to-all tables");
static_assert(kWinA2aOff + kMaxBlocks * kMaxRanks * 16 <= kRsArriveOff, "all-to-all tables overlap the arrivals");
static_assert(kRsPairFreeOff + 4 <= kCtrlHeader, "pair reduce-scatter counters leave the header");
constexpr unsigned char kGuardByte = 0xA5;  // fill of the debug guard regions (VCCL_GUARDS=1)

constexpr size_t kLLMaxBytes = 1 << 20;                 // largest LL payload per source rank
constexpr size_t kLLSlotBytes = 2 * kLLMaxBytes;        // LL lines carry 8 payload bytes per 16
constexpr size_t kLLOff = kCtrlHeader;                  // [parity][src rank][slot]
constexpr size_t kLLBytes = 2 * kMaxRanks * kLLSlotBytes;
constexpr size_t kLLResOff = kLLOff + kLLBytes;         // second LL hop (two-shot LL), same shape

constexpr size_t kP2pSlotBytes = 512 << 10;
constexpr size_t kP2pOff = kLLResOff + kLLBytes;        // [src rank][channel][slot]
constexpr size_t kP2pBytes = size_t(kMaxRanks) * kMaxChannels * kP2pSlots * kP2pSlotBytes;
constexpr size_t kCtrlBytes = kP2pOff + kP2pBytes;

// Status words (host-mapped): [0] error code, [1] where, [2] rank, [3] detail.
enum : uint32_t { kOk = 0, kErrTimeout = 1, kErrAborted = 2, kErrBadArg = 3, kErrCapacity = 4 };

struct DevComm {
  int rank;
  int nranks;
  char* ctrl[kMaxRanks];  // every rank's ctrl allocation, mapped here
  char* data[kMaxRanks];  // every rank's data allocation, mapped here
  char* mcData;           // multicast address of the data allocations, or null
  size_t dataBytes;
  char* fused[kMaxRanks]; // every rank's fused-op region (GEMM+RS, AG+GEMM)
  size_t fusedBytes;
  char* moe[kMaxRanks];   // every rank's MoE dispatch/combine region (allocated on first use)
  size_t moeBytes;
  uint32_t* status;              // host-mapped, written by kernels
  const uint32_t* abortWord;     // host-mapped, written by vcclCommAbort
  uint64_t timeoutNs;
};

__device__ __forceinline__ uint64_t globalTimerNs() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ldAcquireSys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ldAcquireSys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void stRelaxedSys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void stReleaseSys64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fenceSys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// Release increment of a counter another GPU (sys) or this GPU (gpu) polls.
__device__ __forceinline__ void redAddReleaseSys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void redAddReleaseGpu(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fenceProxyAlias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Record the first failure.  Status lives in host-mapped memory: plain
// volatile stores, first writer wins.
__device__ __forceinline__ void recordFailure(const DevComm& c, uint32_t code, uint32_t where,
                                              uint32_t detail) {
  volatile uint32_t* s = c.status;
  if (atomicCAS(c.status, 0u, code) == 0u) {
    s[1] = where;
    s[2] = static_cast<uint32_t>(c.rank);
    s[3] = detail;
  }
  __threadfence_system();
}

// Called every few hundred polls of a wait.  The abort word lives in host
// memory, so each read of it crosses PCIe; with hundreds of threads of a
// persistent kernel waiting at once those reads would keep the bus busy and
// slow every poll down.  A wait therefore reads it only once it is older than
// 20 us, and then on about one call in eight (a hash of the time decides),
// which still notices vcclCommAbort within a few milliseconds.
__device__ __forceinline__ bool shouldGiveUp(const DevComm& c, uint64_t start, uint32_t where,
                                             uint32_t detail) {
  const uint64_t now = globalTimerNs();
  if (now - start > c.timeoutNs) {
    recordFailure(c, kErrTimeout, where, detail);
    return true;
  }
  if (now - start > 20000u && ((now * 0x9E3779B97F4A7C15ull) >> 61) == 0u &&
      *reinterpret_cast<const volatile uint32_t*>(c.abortWord) != 0u) {
    recordFailure(c, kErrAborted, where, detail);
    return true;
  }
  return false;
}

__device__ __forceinline__ uint32_t ldRelaxedSys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spin until *flag - target >= 0 (wrapping compare), then acquire.  Polls
// with relaxed loads and fences once.  False on timeout/abort.
__device__ __forceinline__ bool waitAtLeast(const DevComm& c, const uint32_t* flag, uint32_t target,
                                            uint32_t where, uint32_t detail) {
  if (static_cast<int32_t>(ldRelaxedSys(flag) - target) < 0) {
    const uint64_t start = globalTimerNs();
    for (uint32_t spin = 1;; ++spin) {
      if (static_cast<int32_t>(ldRelaxedSys(flag) - target) >= 0) break;
      if ((spin & 255u) == 0u && shouldGiveUp(c, start, where, detail)) return false;
    }
  }
  fenceSys();
  return true;
}
__device__ __forceinline__ void stReleaseSys32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Spin until *flag - target >= 0, then acquire.  The spin polls with
// relaxed loads and the final check is one acquire load: the flags are
// monotonic counters bumped by release RMWs, so the acquire load reads a
// value of the same release sequence and synchronises with its writer.
// Acquire loads in the spin itself were measured to disturb the memory
// system when hundreds of threads of a persistent kernel wait at once.
// backoffNs > 0 sleeps between polls after the first few hundred (for
// waits that are expected to be long, e.g. a GEMM waiting for remote data).
// False on timeout/abort.
__device__ __forceinline__ bool waitAcquire(const DevComm& c, const uint32_t* flag, uint32_t target, uint32_t where,
                                            uint32_t detail, uint32_t backoffNs = 0) {
  if (static_cast<int32_t>(ldAcquireSys(flag) - target) >= 0) return true;
  const uint64_t start = globalTimerNs();
  for (uint32_t spin = 1;; ++spin) {
    if (static_cast<int32_t>(ldRelaxedSys(flag) - target) >= 0) {
      (void)ldAcquireSys(flag);
      return true;
    }
    if ((spin & 255u) == 0u && shouldGiveUp(c, start, where, detail)) return false;
    if (backoffNs != 0u && spin > 256u) __nanosleep(backoffNs);
  }
}

__device__ __forceinline__ bool waitAtLeast64(const DevComm& c, const uint64_t* flag,
                                              uint64_t target, uint32_t where, uint32_t detail) {
  if (ldAcquireSys64(flag) >= target) return true;
  const uint64_t start = globalTimerNs();
  for (uint32_t spin = 1;; ++spin) {
    if (ldAcquireSys64(flag) >= target) return true;
    if ((spin & 255u) == 0u && shouldGiveUp(c, start, where, detail)) return false;
  }
}

template <typename T>
__device__ __forceinline__ T* ctrlAt(const DevComm& c, int rank, size_t off) {
  return reinterpret_cast<T*>(c.ctrl[rank] + off);
}

// All threads of the block call this.  Block `blk` of this rank meets block
// `blk` of every other rank.  Writes made by the block before the call are
// visible to the peers' blocks after it.  Returns false if the block must
// abandon the kernel (timeout or abort recorded).
__device__ __forceinline__ bool blockBarrier(const DevComm& c, int blk, uint32_t where,
                                             size_t epochOff = kBarEpochOff,
                                             size_t flagsOff = kBarFlagsOff) {
  __shared__ uint32_t sEpoch;
  __shared__ int sFailed;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* ep = ctrlAt<uint32_t>(c, c.rank, epochOff) + blk;
    sEpoch = *ep + 1u;
    *ep = sEpoch;
    sFailed = 0;
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < c.nranks) {
    // Release store / acquire poll: measured about half the latency of a
    // fence.acq_rel.sys on each side.  The release is cumulative over the
    // block's writes ordered before it by the bar.sync above.
    const uint32_t e = sEpoch;
    stReleaseSys32(ctrlAt<uint32_t>(c, t, flagsOff) + blk * kMaxRanks + c.rank, e);
    const uint32_t* mine = ctrlAt<uint32_t>(c, c.rank, flagsOff) + blk * kMaxRanks + t;
    if (!waitAcquire(c, mine, e, where, static_cast<uint32_t>(t))) sFailed = 1;
  }
  __syncthreads();
  return sFailed == 0;
}

// ---- 16-byte vector memory helpers -----------------------------------------
__device__ __forceinline__ uint4 ldCG(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void stG(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

}  // namespace dev
}  // namespace vccl
