// SPDX-License-Identifier: Apache-2.0
// Host side of the tcgen05 GEMM: tensor-map construction, tile-width
// selection and the plain / SiLU*mul entry points.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

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

int* errorFlag() {
  static int* p = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaMalloc(&p, sizeof(int) * 64);
    cudaMemset(p, 0, sizeof(int) * 64);
  });
  return p;
}

}  // namespace gemm
}  // namespace vccl

using namespace vccl;

extern "C" {

vcclResult_t vcclGemmBf16(const void* A, const void* W, void* C, int M, int N, int K, vcclStream_t stream) {
  if (!A || !W || !C || M <= 0 || N <= 0 || K <= 0 || (N % 16) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  gemm::EpiStore epi{static_cast<__nv_bfloat16*>(C), N};
  cudaError_t e = gemm::launchGemm(A, W, M, N, K, epi, gemm::NoHooks{}, reinterpret_cast<cudaStream_t>(stream),
                                   static_cast<int>(gemm::envLongGemm("VCCL_GEMM_BN")), 0);
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
