// SPDX-License-Identifier: Apache-2.0
// Host side of the tcgen05 GEMM: tensor-map construction, tile-width
// selection and the plain / SiLU*mul entry points.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common/log.h"
#include "fused/gemm_launch.cuh"
#include "runtime/cudrv.h"
#include "vccl_tp.h"

namespace vccl {
namespace gemm {

bool makeMapKMajor(CUtensorMap* map, const void* base, int rows, int K, int boxRows) {
  const DriverApi* d = driverApi();
  if (d == nullptr || d->tensorMapEncodeTiled == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (K % 8) != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(boxRows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = d->tensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                       strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    VERR("cuTensorMapEncodeTiled failed: %s", cuErrorText(r));
    return false;
  }
  return true;
}

int smCount() {
  static int n = [] {
    int dev = 0, c = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    return c;
  }();
  return n;
}

int pickBN(int M, int N) {
  const int sms = smCount();
  const int tm = (M + kBM - 1) / kBM;
  for (int bn : {256, 128, 64}) {
    const int tiles = tm * ((N + bn - 1) / bn);
    if (tiles >= sms) return bn;
  }
  return 32;
}

SplitPlan planSplitK(int M, int N, int K) {
  const int sms = smCount();
  const int tilesM = (M + kBM - 1) / kBM;
  const int numK = (K + kBK - 1) / kBK;
  const int tiles = tilesM * ((N + 127) / 128);
  if (tilesM > 2 || tiles * 2 > sms) return {0, 1};
  int splits = sms / tiles;
  if (splits > numK / 4) splits = numK / 4;  // at least 4 k-blocks per split
  if (splits > 16) splits = 16;
  if (splits < 2) return {0, 1};
  return {128, splits};
}

namespace {
__global__ void __launch_bounds__(256) splitReduceKernel(const float4* ws, int splits, size_t n4, size_t stride4,
                                                         uint2* out) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float4 a = ws[i];
    for (int sp = 1; sp < splits; sp++) {
      const float4 b = ws[sp * stride4 + i];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    out[i] = make_uint2(packBf16(a.x, a.y), packBf16(a.z, a.w));
  }
}
}  // namespace

cudaError_t launchSplitReduce(const float* ws, int splits, size_t elems, void* out, cudaStream_t st) {
  const size_t n4 = elems / 4;
  size_t blocks = (n4 + 255) / 256;
  if (blocks > static_cast<size_t>(smCount()) * 4) blocks = static_cast<size_t>(smCount()) * 4;
  if (blocks == 0) blocks = 1;
  splitReduceKernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(reinterpret_cast<const float4*>(ws), splits, n4,
                                                                   n4, static_cast<uint2*>(out));
  return cudaGetLastError();
}

// Split-K scratch, cached per (device, stream) so steady-state calls
// allocate nothing: calls on one stream are ordered, and calls on different
// streams use different buffers.  A call that needs more than the cached
// size waits for its stream, frees the old buffer and allocates a larger one.
// Not used while the stream is being captured (see vcclGemmBf16).
float* splitScratch(cudaStream_t st, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto& e = cache[{dev, st}];
  if (e.second < bytes) {
    if (e.first != nullptr) {
      cudaStreamSynchronize(st);
      cudaFree(e.first);
      e = {nullptr, 0};
    }
    const size_t sz = (bytes + (1u << 20) - 1) / (1u << 20) * (1u << 20);
    void* p = nullptr;
    if (cudaMalloc(&p, sz) != cudaSuccess) return nullptr;
    e = {p, sz};
  }
  return static_cast<float*>(e.first);
}

// One abort flag per device (kernels only ever write their own device's).
int* errorFlag() {
  static std::mutex mu;
  static int* flags[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  std::lock_guard<std::mutex> lock(mu);
  if (flags[dev] == nullptr) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int) * 64) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int) * 64);
    flags[dev] = p;
  }
  return flags[dev];
}

}  // namespace gemm
}  // namespace vccl

using namespace vccl;

extern "C" {

vcclResult_t vcclGemmBf16(const void* A, const void* W, void* C, int M, int N, int K, vcclStream_t stream) {
  if (!A || !W || !C || M <= 0 || N <= 0 || K <= 0 || (N % 16) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int bnEnv = static_cast<int>(gemm::envLongGemm("VCCL_GEMM_BN"));
  const char* sk = std::getenv("VCCL_GEMM_SPLITK");
  const gemm::SplitPlan plan = (bnEnv > 0 || (sk && sk[0] == '0')) ? gemm::SplitPlan{0, 1} : gemm::planSplitK(M, N, K);
  if (plan.splits > 1) {
    // Decode shapes: split K across more CTAs.  The fp32 partials live in a
    // scratch buffer cached for this stream; while the stream is being
    // captured into a CUDA graph they come from a stream-ordered allocation
    // instead (a memory node of the graph), since nothing may be allocated
    // synchronously then.
    const size_t elems = static_cast<size_t>(M) * N;
    const size_t bytes = elems * plan.splits * sizeof(float);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    const bool capturing = cap != cudaStreamCaptureStatusNone;
    float* ws = nullptr;
    if (capturing) {
      if (cudaMallocAsync(reinterpret_cast<void**>(&ws), bytes, st) != cudaSuccess) ws = nullptr;
    } else {
      ws = gemm::splitScratch(st, bytes);
    }
    if (ws == nullptr) {
      VERR("vcclGemmBf16: cannot allocate %zu bytes of split-K scratch", bytes);
      return vcclSystemError;
    }
    gemm::EpiPartialF32 epi{ws, N, elems};
    cudaError_t e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, st, plan.bn, 0, plan.splits);
    if (e == cudaSuccess) e = gemm::launchSplitReduce(ws, plan.splits, elems, C, st);
    if (capturing) cudaFreeAsync(ws, st);
    if (e != cudaSuccess) {
      VERR("vcclGemmBf16 (split-K %d): %s", plan.splits, cudaGetErrorString(e));
      return vcclInvalidArgument;
    }
    return vcclSuccess;
  }
  gemm::EpiStore epi{static_cast<__nv_bfloat16*>(C), N};
  cudaError_t e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, st, bnEnv, 0);
  if (e != cudaSuccess) {
    VERR("vcclGemmBf16: %s", cudaGetErrorString(e));
    return vcclInvalidArgument;
  }
  return vcclSuccess;
}

vcclResult_t vcclGemmSiluMul(const void* A, const void* W, void* H, int M, int N, int K, vcclStream_t stream) {
  if (!A || !W || !H || M <= 0 || N <= 0 || K <= 0 || (N % 32) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  gemm::EpiSiluMul epi{static_cast<__nv_bfloat16*>(H), N / 2};
  cudaError_t e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, reinterpret_cast<cudaStream_t>(stream),
                                   static_cast<int>(gemm::envLongGemm("VCCL_GEMM_BN")), 0);
  if (e != cudaSuccess) {
    VERR("vcclGemmSiluMul: %s", cudaGetErrorString(e));
    return vcclInvalidArgument;
  }
  return vcclSuccess;
}

}  // extern "C"
