// Shared helpers for the loraforge_b200 sm_100a kernels and their C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>
#include <utility>

#include "../../include/loraforge_b200.h"

namespace lfb {

// ---------------------------------------------------------------- host errors
// The message of the last failure on this host thread (lf_last_error_string).
std::string& last_error();

inline int fail(int code, const char* message) {
  last_error() = message;
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    last_error() = std::string(what) + ": " + cudaGetErrorString(err);
    return LF_E_CUDA;
  }
  return LF_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- bf16 bits
// BF16 is handled as raw 16-bit patterns so that rounding is explicit.
__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits) {
  return __uint_as_float(bits << 16);
}

// Round-to-nearest-even FP32 -> BF16 bit pattern; NaN/Inf exponents pass through
// truncated (the behaviour of the reference's round_bf16,
// src/loraforge/ops/csrc/lora_rows.cu:27-33).
__device__ __forceinline__ uint32_t float_to_bf16_bits(float value) {
  uint32_t u = __float_as_uint(value);
  if ((u & 0x7f800000u) != 0x7f800000u) u += 0x7fffu + ((u >> 16) & 1u);
  return u >> 16;
}

__device__ __forceinline__ float round_through_bf16(float value) {
  return bf16_bits_to_float(float_to_bf16_bits(value));
}

// Unpack 8 BF16 values held in a 16-byte vector into FP32.
__device__ __forceinline__ void unpack_bf16x8(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// ---------------------------------------------------------------- generic element types
// Storage types for the dtype-generic (BGMV / vLLM) kernels.
struct f32_t {
  using storage = float;
  __device__ __forceinline__ static float load(const float* p) { return *p; }
  __device__ __forceinline__ static float to_float(float v) { return v; }
  __device__ __forceinline__ static float from_float(float v) { return v; }
};
struct f16_t {
  using storage = __half;
  __device__ __forceinline__ static float to_float(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_float(float v) { return __float2half_rn(v); }
};
struct bf16_t {
  using storage = __nv_bfloat16;
  __device__ __forceinline__ static float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float v) { return __float2bfloat16_rn(v); }
};

// Round an FP32 value through the element type (used for "delta rounded to the
// activation dtype before the base add" semantics).
template <typename T>
__device__ __forceinline__ float round_through(float v) {
  return T::to_float(T::from_float(v));
}

// Unpack 8 values of a 16-bit element type held in a 16-byte vector into FP32 (exact).
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float* out);
template <>
__device__ __forceinline__ void unpack8<bf16_t>(const uint4& v, float* out) {
  unpack_bf16x8(v, out);
}
template <>
__device__ __forceinline__ void unpack8<f16_t>(const uint4& v, float* out) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

template <typename I>
__device__ __forceinline__ int load_index(const void* base, int64_t i) {
  return static_cast<int>(reinterpret_cast<const I*>(base)[i]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

}  // namespace lfb
