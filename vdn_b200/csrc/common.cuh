// Shared helpers for the vdn_b200 C-ABI library: status codes, the thread-local
// error message, bf16 bit helpers and launch checking.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/vdn_b200.h"

namespace vdn {

// Records a printf-style message for vdn_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

#define VDN_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::vdn::set_error(VDN_ERR_VALUE, __VA_ARGS__); \
  } while (0)

#define VDN_CUDA_TRY(expr)                                                          \
  do {                                                                              \
    cudaError_t err__ = (expr);                                                     \
    if (err__ != cudaSuccess)                                                       \
      return ::vdn::set_error(VDN_ERR_RUNTIME, "%s failed: %s", #expr,              \
                              cudaGetErrorString(err__));                           \
  } while (0)

#define VDN_LAUNCH_CHECK(name)                                                      \
  do {                                                                              \
    cudaError_t err__ = cudaGetLastError();                                         \
    if (err__ != cudaSuccess)                                                       \
      return ::vdn::set_error(VDN_ERR_RUNTIME, "%s launch failed: %s", name,        \
                              cudaGetErrorString(err__));                           \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// Round to nearest even, finite inputs (the hardware conversion).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Unpacks the 8 bf16 values of a 16-byte vector.
__device__ __forceinline__ void unpack8(const uint4& v, float* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = __uint_as_float(w[i] << 16);
    out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                    pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

}  // namespace vdn
