// Shared device helpers for the OLMoE sparse-MoE kernels (sm_100a).
//
// Arithmetic that must be bit-exact with the CPU oracle (RMSNorm, router,
// softmax, rank, combine) uses explicitly rounded intrinsics (__fmul_rn,
// __fadd_rn, __fdiv_rn, __fsqrt_rn) so that no multiply-add contraction or
// fast-math substitution can change a result.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/trifuse_b200.h"

namespace tf {

// ---------------------------------------------------------------------------
// activation dtype traits

template <typename T>
struct Act;

template <>
struct Act<__half> {
  static constexpr tf_dtype kDtype = TF_DTYPE_F16;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float f) { return __float2half_rn(f); }
};

template <>
struct Act<__nv_bfloat16> {
  static constexpr tf_dtype kDtype = TF_DTYPE_BF16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float f) { return __float2bfloat16_rn(f); }
};

template <typename T>
__device__ __forceinline__ float to_f(T v) { return Act<T>::to_f(v); }
template <typename T>
__device__ __forceinline__ T from_f(float f) { return Act<T>::from_f(f); }
// Round an fp32 value to the activation dtype and return it as fp32.
template <typename T>
__device__ __forceinline__ float round_act(float f) { return Act<T>::to_f(Act<T>::from_f(f)); }

__device__ __forceinline__ float f16_to_f(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

// Eight packed activation values (16 bytes) -> fp32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float* out) {
  const T* p = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = to_f(p[i]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* in) {
  uint4 v;
  T* p = reinterpret_cast<T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = from_f<T>(in[i]);
  return v;
}

// ---------------------------------------------------------------------------
// memory

// Streaming 16-byte read of weights: read once, do not keep in L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ld_v4(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// ---------------------------------------------------------------------------
// fixed-order reductions

// xor butterfly over a warp with offsets 16, 8, 4, 2, 1: every lane ends with
// the same value because fp32 addition is commutative.
__device__ __forceinline__ float warp_sum_butterfly(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Sum of squares of an 8-element chunk in order: acc = acc + x*x from 0.
__device__ __forceinline__ float chunk_sumsq8(const float* x) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, __fmul_rn(x[i], x[i]));
  return acc;
}

// 1 / sqrt(sumsq / width + eps) with IEEE-rounded steps.
__device__ __forceinline__ float rms_scale(float sumsq, int width, float eps) {
  const float mean = __fdiv_rn(sumsq, (float)width);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

}  // namespace tf
