// SPDX-License-Identifier: Apache-2.0
// Kernel argument structures shared by host launchers and device code.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "kernels/device_common.cuh"

namespace vccl {
namespace dev {

enum Where : uint32_t {
  kWhereStart = 1,
  kWhereLL = 2,
  kWherePush = 3,
  kWhereReduce = 4,
  kWhereNvls = 5,
  kWhereGather = 6,
  kWhereP2pSend = 7,
  kWhereP2pRecv = 8,
  kWhereFused = 9,
  kWhereMoe = 10,
  kWhereWindow = 11,
};

struct CollArgs {
  const char* send;
  char* recv;
  size_t count;   // AR/Reduce/Bcast: elements; AG: sendcount; RS: recvcount
  int root;       // Reduce/Bcast root; -1 for all-reduce
  int premul;     // scale own contribution by `scalar`
  int avg;        // post-scale by 1/nranks
  double scalar;
};

// Collectives on registered windows (csrc/kernels/window.cuh).
struct WinDesc {
  uint64_t sendOff;
  uint64_t recvOff;
  uint64_t count;
  double scalar;  // PreMulSum factor of this rank's contribution (1 otherwise)
};
static_assert(sizeof(WinDesc) * kMaxBlocks <= 8192, "window descriptors fit their ctrl range");

struct WinArgs {
  const char* send[kMaxRanks];  // every rank's send buffer in this address space ([rank] = own)
  char* recv[kMaxRanks];        // every rank's receive buffer ([rank] = own)
  const char* mcSend;           // multicast address of the send buffers, or null
  char* mcRecv;                 // multicast address of the receive buffers, or null
  uint64_t sendOff;             // offsets inside the windows (agreement check)
  uint64_t recvOff;
  size_t count;                 // all-reduce: elements; all-gather: bytes per rank; reduce-scatter: recvcount
  int premul;
  int avg;
  double scalar;
};

// Element counts and displacements of one rank's all-to-all(v) call.
struct A2aTable {
  uint64_t sc[kMaxRanks], sd[kMaxRanks], rc[kMaxRanks], rd[kMaxRanks];
};

constexpr int kMaxP2pOps = 160;
constexpr int kMaxP2pWork = 160;
enum P2pKind : int { kP2pSend = 0, kP2pRecv = 1, kP2pCopy = 2 };

struct P2pOpDesc {
  char* dst;        // recv buffer (recv/copy)
  const char* src;  // send buffer (send/copy)
  size_t bytes;
  int peer;
  int kind;
};
struct P2pWork {
  int16_t peer;
  int8_t kind;
  int8_t ch;
};
struct P2pPlan {
  int nops;
  int nwork;
  P2pOpDesc ops[kMaxP2pOps];
  P2pWork work[kMaxP2pWork];
};

__host__ __device__ __forceinline__ int p2pChannels(size_t bytes) {
  size_t ch = bytes / (1u << 20);
  if (ch < 1) ch = 1;
  if (ch > static_cast<size_t>(kMaxChannels)) ch = kMaxChannels;
  return static_cast<int>(ch);
}

}  // namespace dev
}  // namespace vccl
