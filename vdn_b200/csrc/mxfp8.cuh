// MXFP8 element rules shared by the quantisers, the scatter kernels and GEMM
// epilogues: the E8M0 scale rule, E4M3 conversion, the SWIZZLE_32_4_4 scale
// address and the GELU forms (reference src/models/ops/mxfp8_quant.py:40-74,
// src/models/ops/mxfp8_kernels.py:24-58).
#pragma once

#include "common.cuh"

#include <string.h>

namespace vdn {

// E8M0 exponent rule on the bit pattern of a non-negative fp32 amax.
// Returns the scale byte and writes the exact multiplier 2^-e.
__host__ __device__ __forceinline__ uint32_t e8m0_from_amax_bits(uint32_t ab, float* inv) {
  const int biased = (int)((ab >> 23) & 255u);
  const int e0 = biased - 135;
  const uint32_t thr = ((uint32_t)biased << 23) | 0x600000u;
  int e = e0 + (ab > thr ? 1 : 0);  // positive floats order like their bit patterns
  if (e < -127) e = -127;
  const uint32_t inv_bits = (uint32_t)(127 - e) << 23;
  float f;
  memcpy(&f, &inv_bits, 4);
  *inv = f;
  return (uint32_t)(e + 127);
}

// fp32 -> float8_e4m3fn, round to nearest even, two at a time (hi -> upper byte).
__device__ __forceinline__ uint16_t e4m3x2(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  // byte 0 = a, byte 1 = b, byte 2 = c, byte 3 = d (little-endian row order)
  return (uint32_t)e4m3x2(b, a) | ((uint32_t)e4m3x2(d, c) << 16);
}

__device__ __forceinline__ int64_t scale_offset(int64_t r, int64_t c, int64_t kp) {
  return ((r >> 7) * (kp >> 7) + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3);
}

enum Act { ACT_NONE = 0, ACT_GELU_TANH = 1, ACT_GELU_ERF = 2, ACT_SWIGLU = 3 };

// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), with
// tanh(u) = 1 - 2 / (exp(2u) + 1) evaluated by the hardware exponential and a
// fast division (a handful of instructions, so the GEMM epilogue that fuses it
// stays small).  Saturates correctly: exp overflow gives tanh = 1, underflow -1.
// The result is rounded to bf16 by every caller; the fp32 error (a few ulp)
// moves that rounding only for values within a few fp32 ulp of a bf16 tie.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float u = k0 * (x + 0.044715f * x * x * x);
  const float t = 1.0f - __fdividef(2.0f, __expf(2.0f * u) + 1.0f);
  return 0.5f * x * (1.0f + t);
}

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
}

}  // namespace vdn
