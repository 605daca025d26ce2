// SPDX-License-Identifier: Apache-2.0
// Datatype / reduction dispatch for the launchers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "kernels/dtypes.cuh"
#include "vccl.h"

#define VCCL_TYPE_CASE(enumv, TY, ...) \
  case enumv: {                        \
    using T = TY;                      \
    __VA_ARGS__;                       \
  } break;

#define VCCL_DISPATCH_TYPE(dt, ...)                                   \
  switch (dt) {                                                       \
    VCCL_TYPE_CASE(vcclInt8, int8_t, __VA_ARGS__)                     \
    VCCL_TYPE_CASE(vcclUint8, uint8_t, __VA_ARGS__)                   \
    VCCL_TYPE_CASE(vcclInt32, int32_t, __VA_ARGS__)                   \
    VCCL_TYPE_CASE(vcclUint32, uint32_t, __VA_ARGS__)                 \
    VCCL_TYPE_CASE(vcclInt64, int64_t, __VA_ARGS__)                   \
    VCCL_TYPE_CASE(vcclUint64, uint64_t, __VA_ARGS__)                 \
    VCCL_TYPE_CASE(vcclFloat16, __half, __VA_ARGS__)                  \
    VCCL_TYPE_CASE(vcclFloat32, float, __VA_ARGS__)                   \
    VCCL_TYPE_CASE(vcclFloat64, double, __VA_ARGS__)                  \
    VCCL_TYPE_CASE(vcclBfloat16, __nv_bfloat16, __VA_ARGS__)          \
    VCCL_TYPE_CASE(vcclFloat8e4m3, __nv_fp8_e4m3, __VA_ARGS__)        \
    VCCL_TYPE_CASE(vcclFloat8e5m2, __nv_fp8_e5m2, __VA_ARGS__)        \
    default:                                                          \
      return cudaErrorInvalidValue;                                   \
  }

// (datatype, reduction) pairs the switch can reduce with multimem.ld_reduce
// (dev::HasMultimem): binds T and K for the body; anything else returns
// cudaErrorInvalidValue.  Used where nvlsSupports() has already been checked.
#define VCCL_DISPATCH_MULTIMEM(dt, op, ...)                              \
  switch (dt) {                                                          \
    case vcclFloat32: {                                                  \
      using T = float;                                                   \
      constexpr int K = vccl::dev::kSum;                                 \
      if ((op) != K) return cudaErrorInvalidValue;                       \
      __VA_ARGS__;                                                       \
    } break;                                                             \
    case vcclBfloat16: {                                                 \
      using T = __nv_bfloat16;                                           \
      VCCL_DISPATCH_OP(op, {                                             \
        if constexpr (vccl::dev::HasMultimem<T, K>::value) {             \
          __VA_ARGS__;                                                   \
        } else {                                                         \
          return cudaErrorInvalidValue;                                  \
        }                                                                \
      })                                                                 \
    } break;                                                             \
    case vcclFloat16: {                                                  \
      using T = __half;                                                  \
      VCCL_DISPATCH_OP(op, {                                             \
        if constexpr (vccl::dev::HasMultimem<T, K>::value) {             \
          __VA_ARGS__;                                                   \
        } else {                                                         \
          return cudaErrorInvalidValue;                                  \
        }                                                                \
      })                                                                 \
    } break;                                                             \
    default:                                                             \
      return cudaErrorInvalidValue;                                      \
  }

#define VCCL_OP_CASE(v, ...)    \
  case v: {                     \
    constexpr int K = v;        \
    __VA_ARGS__;                \
  } break;

#define VCCL_DISPATCH_OP(op, ...)           \
  switch (op) {                             \
    VCCL_OP_CASE(0, __VA_ARGS__)            \
    VCCL_OP_CASE(1, __VA_ARGS__)            \
    VCCL_OP_CASE(2, __VA_ARGS__)            \
    VCCL_OP_CASE(3, __VA_ARGS__)            \
    default:                                \
      return cudaErrorInvalidValue;         \
  }
