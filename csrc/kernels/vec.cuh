// 8-wide load/store helpers shared by the row kernels (RMSNorm, embedding,
// softmax-CE): one call moves 8 elements = 16 bytes of bf16/f16 or 32 bytes
// of fp32 and converts to/from fp32 registers.
#pragma once

#include "common.cuh"

namespace uhfs {

template <typename T>
__device__ __forceinline__ float to_float(T x);
template <>
__device__ __forceinline__ float to_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_float<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* f) {
  if constexpr (sizeof(T) == 2) {
    uint4 r = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_float<T>(h[i]);
  } else {
    float4 a = reinterpret_cast<const float4*>(p)[0];
    float4 b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float* f) {
  if constexpr (sizeof(T) == 2) {
    uint4 r;
    T* h = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_float<T>(f[i]);
    *reinterpret_cast<uint4*>(p) = r;
  } else {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// Load 8 elements, each guarded by `col + i < cols` (scalar path for ragged rows).
template <typename T>
__device__ __forceinline__ void load8_guard(const T* p, float* f, int col, int cols, bool vec_ok) {
  if (vec_ok && col + 8 <= cols) {
    load8<T>(p, f);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (col + i < cols) ? to_float<T>(p[i]) : 0.f;
  }
}

template <typename T>
__device__ __forceinline__ void store8_guard(T* p, const float* f, int col, int cols, bool vec_ok) {
  if (vec_ok && col + 8 <= cols) {
    store8<T>(p, f);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (col + i < cols) p[i] = from_float<T>(f[i]);
  }
}

}  // namespace uhfs
