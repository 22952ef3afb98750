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
inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31) == 0; }

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// fp32 -> bf16, round to nearest even (hardware conversion).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Two roundings in one conversion instruction.
__device__ __forceinline__ void round_bf16_pair(float& a, float& b) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(b), "f"(a));
  a = __uint_as_float(p << 16);
  b = __uint_as_float(p & 0xFFFF0000u);
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

// Rounds two floats to bf16 and packs them (lo in the low half), one instruction.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
  return p;
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                    pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// Packs floats that already hold bf16 values (no rounding: a byte permute).
__device__ __forceinline__ uint32_t pack_exact2(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}

__device__ __forceinline__ uint4 pack_exact8(const float* v) {
  return make_uint4(pack_exact2(v[0], v[1]), pack_exact2(v[2], v[3]),
                    pack_exact2(v[4], v[5]), pack_exact2(v[6], v[7]));
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// The hardware's approximate base-2 exponential, reciprocal and square root (one
// MUFU operation each; inputs and outputs below 2^-126 flush to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float sqrt_approx(float x) {
  float r;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Packed pairs of fp32 (sm_100 f32x2 arithmetic: one instruction for two lanes of
// work, each rounded as its scalar counterpart).  f2 holds (lo, hi) in one 64-bit
// register pair.
using f2 = unsigned long long;
__device__ __forceinline__ f2 f2_pack(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(f2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// sigmoid(x) = 1 / (1 + t) for x >= 0 and t / (1 + t) for x < 0, with t = exp(-|x|) in
// (0, 1].  The exponential is one MUFU operation; the divisor y = 1 + t lies in (1, 2],
// so its reciprocal is taken on the FMA pipe: Newton-Raphson division from the textbook
// linear seed 48/17 - 32/17 D for D = y / 2 in (1/2, 1] (relative error <= 1/17, squared
// by each of three steps: below fp32 rounding).  It halves the MUFU / conversion load
// against exp + a hardware reciprocal, at the price of issue slots; the gate GEMM keeps
// it for single columns and takes full chunks in pairs that share one reciprocal.
__device__ __forceinline__ float sigmoid_nr(float x) {
  const float t = __expf(-fabsf(x));
  const float d = 0.5f * (1.0f + t);
  float r = fmaf(-32.0f / 17.0f, d, 48.0f / 17.0f);
  r = fmaf(r, fmaf(-d, r, 1.0f), r);
  r = fmaf(r, fmaf(-d, r, 1.0f), r);
  r = fmaf(r, fmaf(-d, r, 1.0f), r);
  r *= 0.5f;
  return x >= 0.0f ? r : t * r;
}

// Exact three-way bf16 split of eight fp32 values: x = x1 + x2 + x3 with each part
// the round-to-nearest bf16 of what the earlier parts leave (every subtraction is
// exact in fp32, and the three 8-bit significands cover fp32's 24).  What the first
// two parts leave has at most 8 significant bits, so the third part is that residual
// itself (its rounding would be exact; for |x| < 2^-103 the residual is an fp32
// denormal and the part keeps its upper half, an error below 2^-133): two conversions
// per pair, not three.  Each
// conversion's packed output is the part itself; the residuals are taken in f32x2
// pairs.  w[p] holds part p of the eight values as packed bf16 pairs (element 2i in
// the low half).
__device__ __forceinline__ void split3_bf16x8(const float* x, uint32_t (&w)[3][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float a = x[2 * i], b = x[2 * i + 1];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const uint32_t pk = pack_bf16x2(a, b);
      w[p][i] = pk;
      const f2 r = f2_pack(__uint_as_float(pk << 16), __uint_as_float(pk & 0xFFFF0000u));
      f2_unpack(f2_fma(r, f2_pack(-1.0f, -1.0f), f2_pack(a, b)), a, b);
    }
    w[2][i] = pack_exact2(a, b);
  }
}

}  // namespace vdn
