// SPDX-License-Identifier: Apache-2.0
// Element types and reduction functors for the collective kernels.
//
// Covers the reference's reduction unit (reference: src/core/reduce.cc:90-112,
// :234-408) on the device: sum/prod/max/min over i8,u8,i32,u32,i64,u64,f16,
// f32,f64,bf16 plus fp8 e4m3/e5m2.  16- and 8-bit floats accumulate in fp32
// and round once at the end (more accurate than rounding at every pairwise
// step); integers wrap exactly like unsigned C++ arithmetic.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace vccl {
namespace dev {

enum RedKind : int { kSum = 0, kProd = 1, kMax = 2, kMin = 3 };

template <typename T>
struct Elem;  // storage type T -> accumulator type and conversions

#define VCCL_INT_ELEM(T, U)                                                  \
  template <>                                                                \
  struct Elem<T> {                                                           \
    using Acc = T;                                                           \
    using Bits = U;                                                          \
    static constexpr bool kFloat = false;                                    \
    __device__ __forceinline__ static Acc toAcc(T x) { return x; }           \
    __device__ __forceinline__ static T fromAcc(Acc x) { return x; }         \
    __device__ __forceinline__ static Acc add(Acc a, Acc b) {                \
      return static_cast<T>(static_cast<U>(a) + static_cast<U>(b));          \
    }                                                                        \
    __device__ __forceinline__ static Acc mul(Acc a, Acc b) {                \
      return static_cast<T>(static_cast<U>(a) * static_cast<U>(b));          \
    }                                                                        \
  };
VCCL_INT_ELEM(int8_t, uint8_t)
VCCL_INT_ELEM(uint8_t, uint8_t)
VCCL_INT_ELEM(int32_t, uint32_t)
VCCL_INT_ELEM(uint32_t, uint32_t)
VCCL_INT_ELEM(int64_t, unsigned long long)
VCCL_INT_ELEM(uint64_t, unsigned long long)
#undef VCCL_INT_ELEM

template <>
struct Elem<float> {
  using Acc = float;
  static constexpr bool kFloat = true;
  __device__ __forceinline__ static Acc toAcc(float x) { return x; }
  __device__ __forceinline__ static float fromAcc(Acc x) { return x; }
  __device__ __forceinline__ static Acc add(Acc a, Acc b) { return a + b; }
  __device__ __forceinline__ static Acc mul(Acc a, Acc b) { return a * b; }
};
template <>
struct Elem<double> {
  using Acc = double;
  static constexpr bool kFloat = true;
  __device__ __forceinline__ static Acc toAcc(double x) { return x; }
  __device__ __forceinline__ static double fromAcc(Acc x) { return x; }
  __device__ __forceinline__ static Acc add(Acc a, Acc b) { return a + b; }
  __device__ __forceinline__ static Acc mul(Acc a, Acc b) { return a * b; }
};
template <>
struct Elem<__half> {
  using Acc = float;
  static constexpr bool kFloat = true;
  __device__ __forceinline__ static Acc toAcc(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half fromAcc(Acc x) { return __float2half_rn(x); }
  __device__ __forceinline__ static Acc add(Acc a, Acc b) { return a + b; }
  __device__ __forceinline__ static Acc mul(Acc a, Acc b) { return a * b; }
};
template <>
struct Elem<__nv_bfloat16> {
  using Acc = float;
  static constexpr bool kFloat = true;
  __device__ __forceinline__ static Acc toAcc(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 fromAcc(Acc x) { return __float2bfloat16_rn(x); }
  __device__ __forceinline__ static Acc add(Acc a, Acc b) { return a + b; }
  __device__ __forceinline__ static Acc mul(Acc a, Acc b) { return a * b; }
};
template <>
struct Elem<__nv_fp8_e4m3> {
  using Acc = float;
  static constexpr bool kFloat = true;
  __device__ __forceinline__ static Acc toAcc(__nv_fp8_e4m3 x) { return static_cast<float>(x); }
  __device__ __forceinline__ static __nv_fp8_e4m3 fromAcc(Acc x) { return __nv_fp8_e4m3(x); }
  __device__ __forceinline__ static Acc add(Acc a, Acc b) { return a + b; }
  __device__ __forceinline__ static Acc mul(Acc a, Acc b) { return a * b; }
};
template <>
struct Elem<__nv_fp8_e5m2> {
  using Acc = float;
  static constexpr bool kFloat = true;
  __device__ __forceinline__ static Acc toAcc(__nv_fp8_e5m2 x) { return static_cast<float>(x); }
  __device__ __forceinline__ static __nv_fp8_e5m2 fromAcc(Acc x) { return __nv_fp8_e5m2(x); }
  __device__ __forceinline__ static Acc add(Acc a, Acc b) { return a + b; }
  __device__ __forceinline__ static Acc mul(Acc a, Acc b) { return a * b; }
};

template <typename T, int K>
__device__ __forceinline__ typename Elem<T>::Acc combine(typename Elem<T>::Acc a,
                                                         typename Elem<T>::Acc b) {
  if constexpr (K == kSum) return Elem<T>::add(a, b);
  if constexpr (K == kProd) return Elem<T>::mul(a, b);
  if constexpr (K == kMax) return a > b ? a : b;
  if constexpr (K == kMin) return a < b ? a : b;
  return a;
}

// Scale by s (PreMulSum pre-scale, Avg post-scale).  Float types only;
// integer instantiations are never called with scaling enabled.
template <typename T>
__device__ __forceinline__ typename Elem<T>::Acc scaleAcc(typename Elem<T>::Acc a, double s) {
  if constexpr (Elem<T>::kFloat) {
    using Acc = typename Elem<T>::Acc;
    return a * static_cast<Acc>(s);
  } else {
    return a;
  }
}

// A 16-byte pack of elements held in accumulator precision.
template <typename T>
struct Pack {
  static constexpr int N = 16 / sizeof(T);
  using Acc = typename Elem<T>::Acc;
  Acc v[N];

  __device__ __forceinline__ void load(const uint4& raw) {
    union { uint4 u; T e[N]; } cvt;
    cvt.u = raw;
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = Elem<T>::toAcc(cvt.e[i]);
  }
  __device__ __forceinline__ uint4 pack() const {
    union { uint4 u; T e[N]; } cvt;
#pragma unroll
    for (int i = 0; i < N; i++) cvt.e[i] = Elem<T>::fromAcc(v[i]);
    return cvt.u;
  }
  template <int K>
  __device__ __forceinline__ void fold(const uint4& raw) {
    union { uint4 u; T e[N]; } cvt;
    cvt.u = raw;
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = combine<T, K>(v[i], Elem<T>::toAcc(cvt.e[i]));
  }
  __device__ __forceinline__ void scale(double s) {
#pragma unroll
    for (int i = 0; i < N; i++) v[i] = scaleAcc<T>(v[i], s);
  }
};

// Raw 16 bytes, optionally re-encoded after scaling (PreMulSum contribution).
template <typename T>
__device__ __forceinline__ uint4 scaledRaw(const uint4& raw, bool doScale, double s) {
  if (!doScale) return raw;
  Pack<T> p;
  p.load(raw);
  p.scale(s);
  return p.pack();
}

template <typename T>
__device__ __forceinline__ T scaledElem(T x, bool doScale, double s) {
  if (!doScale) return x;
  return Elem<T>::fromAcc(scaleAcc<T>(Elem<T>::toAcc(x), s));
}

}  // namespace dev
}  // namespace vccl
