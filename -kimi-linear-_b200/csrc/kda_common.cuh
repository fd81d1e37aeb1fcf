// kda_common.cuh -- shared device helpers for the KDA kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kda_b200.h"

namespace kda {

// The reference clamps fp16 recurrent outputs to +-FP16_MAX_SAFE
// (kimi_linear/fp16.py:97, applied at kimi_linear/kda.py:217-218).
constexpr float kFp16MaxSafe = 60000.0f;

// ---------------------------------------------------------------------------
// scalar element load / store with conversion to / from fp32
// ---------------------------------------------------------------------------
template <typename T> struct Elt;
template <> struct Elt<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float x) { *p = x; }
};
template <> struct Elt<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float x) { *p = __float2half_rn(x); }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float x) {
    *p = __float2bfloat16_rn(x);
  }
};

template <typename T> __device__ __forceinline__ float ld(const T* p) { return Elt<T>::load(p); }
template <typename T> __device__ __forceinline__ void st(T* p, float x) { Elt<T>::store(p, x); }

// Four consecutive elements -> fp32 (caller guarantees alignment when vec).
template <typename T>
__device__ __forceinline__ void ld4(const T* p, float (&x)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = ld(p + i);
}
template <>
__device__ __forceinline__ void ld4<float>(const float* p, float (&x)[4]) {
  float4 t = *reinterpret_cast<const float4*>(p);
  x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
}
template <>
__device__ __forceinline__ void ld4<__half>(const __half* p, float (&x)[4]) {
  uint2 t = *reinterpret_cast<const uint2*>(p);
  float2 a = __half22float2(*reinterpret_cast<__half2*>(&t.x));
  float2 b = __half22float2(*reinterpret_cast<__half2*>(&t.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
template <>
__device__ __forceinline__ void ld4<__nv_bfloat16>(const __nv_bfloat16* p, float (&x)[4]) {
  uint2 t = *reinterpret_cast<const uint2*>(p);
  float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&t.x));
  float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&t.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}

template <typename T>
__device__ __forceinline__ void st4(T* p, const float (&x)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) st(p + i, x[i]);
}
template <>
__device__ __forceinline__ void st4<float>(float* p, const float (&x)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
}
template <>
__device__ __forceinline__ void st4<__half>(__half* p, const float (&x)[4]) {
  __half2 a = __floats2half2_rn(x[0], x[1]);
  __half2 b = __floats2half2_rn(x[2], x[3]);
  uint2 t;
  t.x = *reinterpret_cast<uint32_t*>(&a);
  t.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = t;
}
template <>
__device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, const float (&x)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(x[2], x[3]);
  uint2 t;
  t.x = *reinterpret_cast<uint32_t*>(&a);
  t.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = t;
}

// Output clamp of the fp16 recurrent path (identity for other types).
template <typename T> __device__ __forceinline__ float clamp_out(float x) { return x; }
template <> __device__ __forceinline__ float clamp_out<__half>(float x) {
  return fminf(fmaxf(x, -kFp16MaxSafe), kFp16MaxSafe);
}

// exp for the decay factors.  PRECISE selects CUDA's expf (fp32 inputs, where
// parity is 1e-5); otherwise the __expf intrinsic, whose documented error
// (2 + 1.16|x| ulp) only grows for arguments whose exp is already negligible.
template <bool PRECISE> __device__ __forceinline__ float dexp(float x) {
  return PRECISE ? expf(x) : __expf(x);
}

}  // namespace kda
