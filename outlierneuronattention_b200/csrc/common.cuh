// Shared device helpers for the HOFA B200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hofa.h"

namespace hofa {

constexpr float kLog2e = 1.4426950408889634f;

// ---- scalar loads of any activation dtype, converted to float --------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Load element `off` of a tensor whose dtype is only known at run time
// (small per-token/per-head side inputs: log_gamma, mix, gla_scale, ...).
__device__ __forceinline__ float ld_any(const void* p, int dtype, int64_t off) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off]);
    case HOFA_DTYPE_F16: return __half2float(reinterpret_cast<const __half*>(p)[off]);
    default: return reinterpret_cast<const float*>(p)[off];
  }
}
__device__ __forceinline__ void st_any(void* p, int dtype, int64_t off, float x) {
  switch (dtype) {
    case HOFA_DTYPE_BF16: reinterpret_cast<__nv_bfloat16*>(p)[off] = __float2bfloat16_rn(x); break;
    case HOFA_DTYPE_F16: reinterpret_cast<__half*>(p)[off] = __float2half_rn(x); break;
    default: reinterpret_cast<float*>(p)[off] = x; break;
  }
}

// ---- 8-element vector loads -------------------------------------------------
// Streaming (read-once) 16-byte load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ void bf16x2_to_f(uint32_t u, float& a, float& b) {
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xffff0000u);
}
__device__ __forceinline__ void f16x2_to_f(uint32_t u, float& a, float& b) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  float2 f = __half22float2(h);
  a = f.x; b = f.y;
}

// Raw storage of 8 elements of T (16 bytes for 2-byte types, 32 for float).
template <typename T> struct Vec8 { uint4 w[sizeof(T) == 4 ? 2 : 1]; };

template <typename T>
__device__ __forceinline__ Vec8<T> ld_vec8(const T* p) {
  Vec8<T> v;
  v.w[0] = ld_stream16(p);
  if constexpr (sizeof(T) == 4) v.w[1] = ld_stream16(reinterpret_cast<const char*>(p) + 16);
  return v;
}
template <typename T>
__device__ __forceinline__ Vec8<T> ld_strided8(const T* p, int64_t stride) {
  Vec8<T> v;
  T tmp[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) tmp[i] = p[i * stride];
  memcpy(&v, tmp, sizeof(tmp));
  return v;
}
template <typename T>
__device__ __forceinline__ Vec8<T> zero_vec8() {
  Vec8<T> v;
#pragma unroll
  for (int i = 0; i < (int)(sizeof(v.w) / sizeof(uint4)); ++i) v.w[i] = make_uint4(0, 0, 0, 0);
  return v;
}

template <typename T>
__device__ __forceinline__ void vec8_to_f(const Vec8<T>& v, float f[8]) {
  if constexpr (sizeof(T) == 4) {
    const float* p = reinterpret_cast<const float*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = p[i];
  } else {
    const uint32_t u[4] = {v.w[0].x, v.w[0].y, v.w[0].z, v.w[0].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) bf16x2_to_f(u[i], f[2 * i], f[2 * i + 1]);
      else f16x2_to_f(u[i], f[2 * i], f[2 * i + 1]);
    }
  }
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

}  // namespace hofa
