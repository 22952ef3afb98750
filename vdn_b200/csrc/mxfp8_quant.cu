// MXFP8 producers for sm_100a: block-32 E4M3 codes with one E8M0 scale per 32
// K-elements, scales stored in the SWIZZLE_32_4_4 layout the tcgen05 block-scaled
// MMA consumes directly (one 512-byte atom = 128 rows x 4 scale columns).
//
// Reference rule (ec-jt/vdn src/models/ops/mxfp8_quant.py:64-73,
// src/models/ops/mxfp8_kernels.py:14-58):
//   e0 = biased_exp(amax) - 135, thr = 1.75 * 2^(e0+8),
//   e = max(e0 + (amax > thr), -127), code = e4m3_rne(x * 2^-e), byte = e + 127.
// The multiply by 2^-e is exact and denormals are never flushed (this file is
// compiled without -ftz), so the codes are bit-identical to the reference.
//
// Kernels here are HBM-bound; one thread owns one 32-element block (64 input
// bytes, 32 code bytes) and lanes 4i..4i+3 pack their scale bytes into one
// 32-bit store, because four consecutive K-blocks of a row are contiguous in
// the swizzled layout.
#include "common.cuh"
#include "mxfp8.cuh"

#include <math.h>
#include <string.h>
#include <algorithm>
#include <cmath>
#include <mutex>
#include <thread>
#include <vector>

namespace vdn {


// Column grouping: logical column j of a row lives at (j / group) * group_stride
// + j % group (group = k, group_stride = k for a plain row).  Used to quantise
// one half of per-head interleaved [softmax | linear] rows without a copy.
// Loads the 32 inputs of block (r, c) as fp32, zero outside [rows, k).
template <bool VEC>
__device__ __forceinline__ void load_block(const uint16_t* __restrict__ x, int64_t row_stride,
                                           int64_t r, int64_t c, int64_t rows, int64_t k,
                                           float* v, int64_t group = 0, int64_t group_stride = 0) {
  const int64_t col0 = c * 32;
  const int64_t phys0 = group ? (col0 / group) * group_stride + col0 % group : col0;
  if (r < rows && VEC && col0 + 32 <= k) {
    const uint4* p = reinterpret_cast<const uint4*>(x + r * row_stride + phys0);
#pragma unroll
    for (int i = 0; i < 4; ++i) unpack8(__ldg(p + i), v + 8 * i);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int64_t col = col0 + i;
      const int64_t phys = group ? (col / group) * group_stride + col % group : col;
      v[i] = (r < rows && col < k) ? bf16_bits_to_f32(x[r * row_stride + phys]) : 0.0f;
    }
  }
}

// One 32-element block: activation, bf16 rounding (when an activation ran), scale,
// codes, and the finite predicate of the inputs and the produced values.
template <int ACT, bool VEC>
__global__ void __launch_bounds__(256) act_quantize_kernel(
    const uint16_t* __restrict__ x, int64_t row_stride, int64_t rows, int64_t k, int64_t rp,
    int64_t kp, uint8_t* __restrict__ q, uint8_t* __restrict__ s, int* __restrict__ nonfinite,
    int64_t group = 0, int64_t group_stride = 0) {
  const int64_t nblk = kp >> 5;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = g < rp * nblk;
  const int64_t r = active ? g / nblk : 0;
  const int64_t c = active ? g - r * nblk : 0;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = 0.0f;
  bool bad = false;
  if (active) {
    load_block<VEC>(x, row_stride, r, c, rows, k, v, group, group_stride);
#pragma unroll
    for (int i = 0; i < 32; ++i) bad |= !isfinite(v[i]);
    if (ACT == ACT_SWIGLU) {
      float gte[32];
      load_block<VEC>(x + k, row_stride, r, c, rows, k, gte);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        bad |= !isfinite(gte[i]);
        // a * (g * sigmoid(g)) rounded to bf16, no contraction (reference
        // src/models/ops/mxfp8_kernels.py:61-74).
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gte[i])));
        v[i] = round_bf16(__fmul_rn(v[i], __fmul_rn(gte[i], sg)));
        bad |= !isfinite(v[i]);
      }
    } else if (ACT == ACT_GELU_TANH || ACT == ACT_GELU_ERF) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v[i] = round_bf16(ACT == ACT_GELU_TANH ? gelu_tanh(v[i]) : gelu_erf(v[i]));
        bad |= !isfinite(v[i]);
      }
    }
  }
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t b = __float_as_uint(v[i]) & 0x7FFFFFFFu;
    amax_bits = b > amax_bits ? b : amax_bits;
  }
  float inv;
  const uint32_t sbyte = e8m0_from_amax_bits(amax_bits, &inv);
  // Pack four scale bytes of c..c+3 (same row: nblk % 4 == 0) into one word.
  const unsigned lane = threadIdx.x & 31;
  uint32_t word = sbyte << (8 * (lane & 3));
  word |= __shfl_xor_sync(0xffffffffu, word, 1);
  word |= __shfl_xor_sync(0xffffffffu, word, 2);
  if (!active) return;
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    packed[i] = e4m3x4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv, v[4 * i + 3] * inv);
  uint4* qp = reinterpret_cast<uint4*>(q + r * kp + c * 32);
  qp[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  qp[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(s + scale_offset(r, c, kp)) = word;
  if (bad && nonfinite) atomicAdd(nonfinite, 1);
}

// RMSNorm * w, AdaLN affine (1 + scale[idx]) and shift[idx], bf16 rounding, then
// MXFP8 of that bf16 value. Rows past `rows` quantise
// exact zeros (reference src/models/ops/mxfp8_kernels.py:86-139).
template <typename WT>
__device__ __forceinline__ void load_weight8(const WT* w, float* out);
template <>
__device__ __forceinline__ void load_weight8<float>(const float* w, float* out) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(w));
  const float4 b = __ldg(reinterpret_cast<const float4*>(w) + 1);
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}
template <>
__device__ __forceinline__ void load_weight8<__nv_bfloat16>(const __nv_bfloat16* w, float* out) {
  unpack8(__ldg(reinterpret_cast<const uint4*>(w)), out);
}

// One warp per (padded) row, eight rows per CTA.  Pass 1 reduces the row's sum
// of squares; pass 2 re-reads the row (L1/L2 resident) one 32-element block per
// lane, applies RMSNorm * w * (1 + scale[idx]) + shift[idx] with the eager bf16
// rounding point, and writes the optional bf16 copy, the E4M3 codes and the
// block's E8M0 byte.  VEC: K % 32 == 0 and every operand 16-byte aligned, so a
// block is four 16-byte loads per operand; otherwise element-wise loads.
template <typename WT, bool VEC>
__global__ void __launch_bounds__(256) prenorm_quantize_kernel(
    const uint16_t* __restrict__ x, int64_t xs, const WT* __restrict__ w,
    const uint16_t* __restrict__ scale, int64_t ss, const uint16_t* __restrict__ shift,
    int64_t ts, const int64_t* __restrict__ idx, int64_t rows, int64_t rp, int64_t k, int64_t kp,
    float eps, uint16_t* __restrict__ y, uint8_t* __restrict__ q, uint8_t* __restrict__ s,
    uint8_t* __restrict__ finite) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rp) return;
  const bool valid = r < rows;
  const uint16_t* xr = x + r * xs;
  float sq = 0.f;
  bool bad = false;
  if (valid) {
    if (VEC) {
      for (int64_t c = lane; c * 32 < k; c += 32) {
        const uint4* src = reinterpret_cast<const uint4*>(xr + c * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v[8];
          unpack8(__ldg(src + j), v);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            sq = fmaf(v[i], v[i], sq);
            bad |= !isfinite(v[i]);
          }
        }
      }
    } else {
      for (int64_t col = lane; col < k; col += 32) {
        const float v = bf16_bits_to_f32(xr[col]);
        sq = fmaf(v, v, sq);
        bad |= !isfinite(v);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float inv_rms = rsqrtf(sq / (float)k + eps);
  const int64_t t = valid ? idx[r] : 0;
  const uint16_t* scr = scale + t * ss;
  const uint16_t* shr = shift + t * ts;
  const int64_t nblk = kp >> 5;
  for (int64_t c = lane; c < nblk; c += 32) {
    float v[32];
    const int64_t col0 = c * 32;
    if (VEC && valid && col0 < k) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float xv[8], wv[8], sc[8], sh[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(xr + col0) + j), xv);
        load_weight8<WT>(w + col0 + 8 * j, wv);
        unpack8(__ldg(reinterpret_cast<const uint4*>(scr + col0) + j), sc);
        unpack8(__ldg(reinterpret_cast<const uint4*>(shr + col0) + j), sh);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[8 * j + i] = __fadd_rn(__fmul_rn(__fmul_rn(__fmul_rn(xv[i], inv_rms), wv[i]),
                                             __fadd_rn(1.0f, sc[i])), sh[i]);
      }
#pragma unroll
      for (int i = 0; i < 32; i += 2) round_bf16_pair(v[i], v[i + 1]);
      if (y) {
        uint4* dst = reinterpret_cast<uint4*>(y + r * k + col0);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = pack_exact8(v + 8 * j);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int64_t col = col0 + i;
        float val = 0.f;
        if (!VEC && valid && col < k) {
          const float xv = bf16_bits_to_f32(xr[col]);
          const float wv = (float)w[col];
          const float sc = bf16_bits_to_f32(scr[col]);
          const float sh = bf16_bits_to_f32(shr[col]);
          val = round_bf16(__fadd_rn(__fmul_rn(__fmul_rn(__fmul_rn(xv, inv_rms), wv),
                                               __fadd_rn(1.0f, sc)), sh));
          if (y) y[r * k + col] = f32_to_bf16_bits(val);
        }
        v[i] = val;
      }
    }
    uint32_t amax_bits = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      bad |= !isfinite(v[i]);
      const uint32_t b = __float_as_uint(v[i]) & 0x7FFFFFFFu;
      amax_bits = b > amax_bits ? b : amax_bits;
    }
    float inv;
    const uint32_t sbyte = e8m0_from_amax_bits(amax_bits, &inv);
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      packed[i] = e4m3x4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv, v[4 * i + 3] * inv);
    uint4* qp = reinterpret_cast<uint4*>(q + r * kp + col0);
    qp[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    qp[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    s[scale_offset(r, c, kp)] = (uint8_t)sbyte;
  }
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) finite[r] = bad ? 0 : 1;
}

// Per-4096-element finite predicate (reference src/models/ops/mxfp8_kernels.py:142-162).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}

// The staged form for K % 32 == 0, aligned operands and K <= kStagedMaxK: four
// rows per CTA, each warp copies its whole row into shared memory with cp.async
// (every byte of the row in flight at once), reduces it, then quantises it with
// four lanes per 32-element block so every global access is a coalesced 16- or
// 8-byte vector and the four E8M0 bytes of blocks c..c+3 leave as one word.
constexpr int64_t kStagedMaxK = 12288;

template <typename WT>
__global__ void __launch_bounds__(128) prenorm_quantize_staged_kernel(
    const uint16_t* __restrict__ x, int64_t xs, const WT* __restrict__ w,
    const uint16_t* __restrict__ scale, int64_t ss, const uint16_t* __restrict__ shift,
    int64_t ts, const int64_t* __restrict__ idx, int64_t rows, int64_t rp, int64_t k, int64_t kp,
    float eps, uint16_t* __restrict__ y, uint8_t* __restrict__ q, uint8_t* __restrict__ s,
    uint8_t* __restrict__ finite) {
  extern __shared__ uint4 staged_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 4 + warp;
  if (r >= rp) return;  // warp-uniform; the kernel has no CTA-wide barrier
  const bool valid = r < rows;
  const int64_t kv = k >> 3;
  uint4* buf = staged_rows + warp * kv;
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(x + r * xs);
    for (int64_t i = lane; i < kv; i += 32) cp_async16(buf + i, src + i);
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
  }
  __syncwarp();
  float sq = 0.f;
  bool bad = false;
  if (valid) {
    for (int64_t i = lane; i < kv; i += 32) {
      float v[8];
      unpack8(buf[i], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sq = fmaf(v[j], v[j], sq);
        bad |= !isfinite(v[j]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float inv_rms = rsqrtf(sq / (float)k + eps);
  const int64_t t = valid ? idx[r] : 0;
  const uint16_t* scr = scale + t * ss;
  const uint16_t* shr = shift + t * ts;
  const int64_t nblk = kp >> 5;
  const int sub = lane & 3;
  for (int64_t c0 = 0; c0 < nblk; c0 += 8) {
    const int64_t c = c0 + (lane >> 2);
    const int64_t col = c * 32 + sub * 8;
    float v[8];
    if (valid && col < k) {
      float xv[8], wv[8], sc[8], sh[8];
      unpack8(buf[col >> 3], xv);
      load_weight8<WT>(w + col, wv);
      unpack8(__ldg(reinterpret_cast<const uint4*>(scr + col)), sc);
      unpack8(__ldg(reinterpret_cast<const uint4*>(shr + col)), sh);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fmul_rn(xv[i], inv_rms), wv[i]), __fadd_rn(1.0f, sc[i])),
                         sh[i]);
#pragma unroll
      for (int i = 0; i < 8; i += 2) round_bf16_pair(v[i], v[i + 1]);
      if (y) *reinterpret_cast<uint4*>(y + r * k + col) = pack_exact8(v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    uint32_t amax_bits = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      bad |= !isfinite(v[i]);
      const uint32_t b = __float_as_uint(v[i]) & 0x7FFFFFFFu;
      amax_bits = b > amax_bits ? b : amax_bits;
    }
    amax_bits = max(amax_bits, __shfl_xor_sync(0xffffffffu, amax_bits, 1));
    amax_bits = max(amax_bits, __shfl_xor_sync(0xffffffffu, amax_bits, 2));
    float inv;
    const uint32_t sbyte = e8m0_from_amax_bits(amax_bits, &inv);
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, sbyte, 4);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, sbyte, 8);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, sbyte, 12);
    if (c < nblk) {
      *reinterpret_cast<uint2*>(q + r * kp + col) =
          make_uint2(e4m3x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv),
                     e4m3x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv));
      // Lanes 0 and 16 hold blocks c = c0 and c0 + 4 (c % 4 == 0; nblk % 4 == 0).
      if ((lane & 15) == 0)
        *reinterpret_cast<uint32_t*>(s + scale_offset(r, c, kp)) = sbyte | b1 << 8 | b2 << 16 | b3 << 24;
    }
  }
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) finite[r] = bad ? 0 : 1;
}

template <typename T, int MODE>
__global__ void finite_parts_kernel(const T* __restrict__ x, int64_t n, uint8_t* __restrict__ parts) {
  const int64_t base = (int64_t)blockIdx.x * 4096;
  int good = 1;
  for (int64_t i = base + threadIdx.x; i < base + 4096 && i < n; i += blockDim.x) {
    if (MODE == 1) good &= ((uint32_t)x[i] & 127u) != 127u;
    else if (MODE == 2) good &= (uint32_t)x[i] != 255u;
    else good &= isfinite((float)x[i]);
  }
  good = __syncthreads_and(good);
  if (threadIdx.x == 0) parts[blockIdx.x] = (uint8_t)good;
}

// ---------------------------------------------------------------- host quantiser
static inline float host_half_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // renormalise the fp16 subnormal
      int e = -1;
      do { ++e; man <<= 1; } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline uint8_t host_e4m3(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint32_t sign = b >> 31;
  const uint32_t exp = (b >> 23) & 0xFF, man = b & 0x7FFFFF;
  uint32_t code;
  if ((int)exp - 120 >= 1) {
    const uint32_t joined = ((exp - 120) << 23) | man;
    code = (joined >> 20) + (((joined & 0xFFFFF) > 0x80000) ||
                             (((joined & 0xFFFFF) == 0x80000) && ((joined >> 20) & 1)));
  } else {
    const uint64_t full = exp ? (man | (1u << 23)) : man;
    const int shift = 141 - (exp ? (int)exp : 1);
    if (shift >= 40) {
      code = 0;
    } else {
      const uint64_t qv = full >> shift, rem = full & ((1ull << shift) - 1), half = 1ull << (shift - 1);
      code = (uint32_t)(qv + ((rem > half) || (rem == half && (qv & 1))));
    }
  }
  return (uint8_t)(code | (sign << 7));
}

static int host_quantize_rows(const void* x, int dtype, int64_t r0, int64_t r1, int64_t rows,
                              int64_t k, int64_t row_stride, int64_t kp, uint8_t* q, uint8_t* s,
                              int* bad) {
  std::vector<float> v(32);
  for (int64_t r = r0; r < r1; ++r) {
    for (int64_t c = 0; c < kp / 32; ++c) {
      uint32_t amax_bits = 0;
      for (int i = 0; i < 32; ++i) {
        const int64_t col = c * 32 + i;
        float f = 0.f;
        if (r < rows && col < k) {
          const int64_t off = r * row_stride + col;
          if (dtype == VDN_DTYPE_F32) {
            f = static_cast<const float*>(x)[off];
          } else if (dtype == VDN_DTYPE_BF16) {
            const uint32_t bits = (uint32_t)static_cast<const uint16_t*>(x)[off] << 16;
            memcpy(&f, &bits, 4);
          } else {
            f = host_half_to_f32(static_cast<const uint16_t*>(x)[off]);
          }
          if (!std::isfinite(f)) { *bad = 1; return 0; }
        }
        v[i] = f;
        uint32_t ab;
        memcpy(&ab, &f, 4);
        ab &= 0x7FFFFFFFu;
        amax_bits = ab > amax_bits ? ab : amax_bits;
      }
      float inv;
      const uint32_t sbyte = e8m0_from_amax_bits(amax_bits, &inv);
      for (int i = 0; i < 32; ++i) q[r * kp + c * 32 + i] = host_e4m3(v[i] * inv);
      s[((r >> 7) * (kp >> 7) + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3)] =
          (uint8_t)sbyte;
    }
  }
  return 0;
}

}  // namespace vdn

using namespace vdn;

extern "C" {

int vdn_mxfp8_padded_shape(int64_t rows, int64_t k, int64_t* rows_padded, int64_t* k_padded) {
  VDN_CHECK_ARG(rows >= 0 && k > 0, "rows must be nonnegative and K positive");
  VDN_CHECK_ARG(rows_padded && k_padded, "output pointers must not be null");
  *rows_padded = (rows + 127) / 128 * 128;
  *k_padded = (k + 127) / 128 * 128;
  return VDN_OK;
}

static int launch_act_quantize(int act, const void* x, int64_t rows, int64_t k, int64_t row_stride,
                               uint8_t* q, uint8_t* s, int* nonfinite, cudaStream_t stream) {
  VDN_CHECK_ARG(rows >= 0 && k > 0, "rows must be nonnegative and K positive");
  if (rows == 0) return VDN_OK;  // zero padded rows: nothing to write
  VDN_CHECK_ARG(q && s, "q and s must not be null");
  VDN_CHECK_ARG(x, "x must not be null");
  const int64_t width = act == ACT_SWIGLU ? 2 * k : k;
  VDN_CHECK_ARG(rows <= 1 || row_stride >= width, "row_stride %lld shorter than the row width %lld",
                (long long)row_stride, (long long)width);
  VDN_CHECK_ARG(aligned16(q) && aligned16(s), "q and s must be 16-byte aligned");
  const int64_t rp = (rows + 127) / 128 * 128, kp = (k + 127) / 128 * 128;
  const bool vec = aligned16(x) && (row_stride % 8 == 0) && (act != ACT_SWIGLU || k % 8 == 0);
  const int64_t threads = rp * (kp / 32);
  const dim3 grid((unsigned)((threads + 255) / 256)), block(256);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
#define VDN_QLAUNCH(A)                                                                       \
  if (vec) act_quantize_kernel<A, true><<<grid, block, 0, stream>>>(xp, row_stride, rows, k, rp, kp, q, s, nonfinite); \
  else act_quantize_kernel<A, false><<<grid, block, 0, stream>>>(xp, row_stride, rows, k, rp, kp, q, s, nonfinite);
  switch (act) {
    case ACT_NONE: VDN_QLAUNCH(ACT_NONE); break;
    case ACT_GELU_TANH: VDN_QLAUNCH(ACT_GELU_TANH); break;
    case ACT_GELU_ERF: VDN_QLAUNCH(ACT_GELU_ERF); break;
    case ACT_SWIGLU: VDN_QLAUNCH(ACT_SWIGLU); break;
    default: return set_error(VDN_ERR_VALUE, "unknown activation %d", act);
  }
#undef VDN_QLAUNCH
  VDN_LAUNCH_CHECK("mxfp8 quantize");
  return VDN_OK;
}

int vdn_mxfp8_quantize(const void* x, int64_t rows, int64_t k, int64_t row_stride, uint8_t* q,
                       uint8_t* s, int* nonfinite, cudaStream_t stream) {
  return launch_act_quantize(ACT_NONE, x, rows, k, row_stride, q, s, nonfinite, stream);
}

int vdn_mxfp8_quantize_grouped(const void* x, int64_t rows, int64_t k, int64_t row_stride,
                               int64_t group, int64_t group_stride, uint8_t* q, uint8_t* s,
                               int* nonfinite, cudaStream_t stream) {
  VDN_CHECK_ARG(rows >= 0 && k > 0, "rows must be nonnegative and K positive");
  VDN_CHECK_ARG(group > 0 && group % 32 == 0 && group_stride >= group,
                "group must be a positive multiple of 32 and group_stride >= group");
  if (rows == 0) return VDN_OK;
  VDN_CHECK_ARG(x && q && s, "null pointer");
  VDN_CHECK_ARG(aligned16(q) && aligned16(s), "q and s must be 16-byte aligned");
  const int64_t rp = (rows + 127) / 128 * 128, kp = (k + 127) / 128 * 128;
  const bool vec = aligned16(x) && row_stride % 8 == 0 && group_stride % 8 == 0;
  const int64_t threads = rp * (kp / 32);
  const dim3 grid((unsigned)((threads + 255) / 256)), block(256);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  if (vec)
    act_quantize_kernel<ACT_NONE, true><<<grid, block, 0, stream>>>(xp, row_stride, rows, k, rp, kp, q, s,
                                                                     nonfinite, group, group_stride);
  else
    act_quantize_kernel<ACT_NONE, false><<<grid, block, 0, stream>>>(xp, row_stride, rows, k, rp, kp, q, s,
                                                                      nonfinite, group, group_stride);
  VDN_LAUNCH_CHECK("mxfp8 quantize (grouped)");
  return VDN_OK;
}

int vdn_mxfp8_act_quantize(int act, const void* x, int64_t rows, int64_t k, int64_t row_stride,
                           uint8_t* q, uint8_t* s, int* nonfinite, cudaStream_t stream) {
  VDN_CHECK_ARG(act >= VDN_ACT_GELU_TANH && act <= VDN_ACT_SWIGLU, "unknown activation %d", act);
  return launch_act_quantize(act, x, rows, k, row_stride, q, s, nonfinite, stream);
}

int vdn_mxfp8_prenorm_quantize(const void* x, int64_t rows, int64_t k, int64_t x_stride,
                               const void* weight, int weight_dtype, float eps, const void* scale,
                               int64_t scale_stride, const void* shift, int64_t shift_stride,
                               const int64_t* indices, void* y, uint8_t* q, uint8_t* s,
                               uint8_t* finite, cudaStream_t stream) {
  VDN_CHECK_ARG(rows >= 0 && k > 0, "rows must be nonnegative and K positive");
  if (rows == 0) return VDN_OK;
  VDN_CHECK_ARG(q && s && finite, "q, s and finite must not be null");
  VDN_CHECK_ARG(rows == 0 || (x && weight && scale && shift && indices), "inputs must not be null");
  VDN_CHECK_ARG(weight_dtype == VDN_DTYPE_F32 || weight_dtype == VDN_DTYPE_BF16,
                "weight must be fp32 or bf16");
  const int64_t rp = (rows + 127) / 128 * 128, kp = (k + 127) / 128 * 128;
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  const bool vec = k % 32 == 0 && aligned16(x) && x_stride % 8 == 0 && aligned16(weight) &&
                   aligned16(scale) && scale_stride % 8 == 0 && aligned16(shift) &&
                   shift_stride % 8 == 0 && (!y || aligned16(y));
  if (vec && k <= kStagedMaxK) {
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
      const int bytes = (int)(4 * kStagedMaxK * 2);
      attr = cudaFuncSetAttribute(prenorm_quantize_staged_kernel<float>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      if (attr == cudaSuccess)
        attr = cudaFuncSetAttribute(prenorm_quantize_staged_kernel<__nv_bfloat16>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    });
    VDN_CUDA_TRY(attr);
    const unsigned sgrid = (unsigned)((rp + 3) / 4);
    const size_t smem = (size_t)4 * k * 2;
#define VDN_PRENORM_STAGED(WT)                                                                 \
  prenorm_quantize_staged_kernel<WT><<<sgrid, 128, smem, stream>>>(                            \
      xp, x_stride, static_cast<const WT*>(weight), static_cast<const uint16_t*>(scale),         \
      scale_stride, static_cast<const uint16_t*>(shift), shift_stride, indices, rows, rp, k, kp, \
      eps, static_cast<uint16_t*>(y), q, s, finite)
    if (weight_dtype == VDN_DTYPE_F32) VDN_PRENORM_STAGED(float);
    else VDN_PRENORM_STAGED(__nv_bfloat16);
#undef VDN_PRENORM_STAGED
    VDN_LAUNCH_CHECK("mxfp8 prenorm quantize");
    return VDN_OK;
  }
  const unsigned grid = (unsigned)((rp + 7) / 8);
#define VDN_PRENORM(WT, V)                                                                     \
  prenorm_quantize_kernel<WT, V><<<grid, 256, 0, stream>>>(                                    \
      xp, x_stride, static_cast<const WT*>(weight), static_cast<const uint16_t*>(scale),         \
      scale_stride, static_cast<const uint16_t*>(shift), shift_stride, indices, rows, rp, k, kp, \
      eps, static_cast<uint16_t*>(y), q, s, finite)
  if (weight_dtype == VDN_DTYPE_F32) {
    if (vec) VDN_PRENORM(float, true);
    else VDN_PRENORM(float, false);
  } else {
    if (vec) VDN_PRENORM(__nv_bfloat16, true);
    else VDN_PRENORM(__nv_bfloat16, false);
  }
#undef VDN_PRENORM
  VDN_LAUNCH_CHECK("mxfp8 prenorm quantize");
  return VDN_OK;
}

int vdn_finite_parts(const void* x, int64_t n, int dtype, int mode, uint8_t* parts,
                     cudaStream_t stream) {
  VDN_CHECK_ARG(n >= 0 && parts, "bad finite_parts arguments");
  VDN_CHECK_ARG(mode >= 0 && mode <= 2, "mode must be 0, 1 or 2");
  if (n == 0) return VDN_OK;
  const unsigned grid = (unsigned)((n + 4095) / 4096);
  if (mode == 1) {
    finite_parts_kernel<uint8_t, 1><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(x), n, parts);
  } else if (mode == 2) {
    finite_parts_kernel<uint8_t, 2><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(x), n, parts);
  } else if (dtype == VDN_DTYPE_F32) {
    finite_parts_kernel<float, 0><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), n, parts);
  } else if (dtype == VDN_DTYPE_BF16) {
    finite_parts_kernel<__nv_bfloat16, 0><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), n, parts);
  } else if (dtype == VDN_DTYPE_F16) {
    finite_parts_kernel<__half, 0><<<grid, 256, 0, stream>>>(static_cast<const __half*>(x), n, parts);
  } else {
    return set_error(VDN_ERR_TYPE, "unsupported dtype %d", dtype);
  }
  VDN_LAUNCH_CHECK("finite_parts");
  return VDN_OK;
}

int vdn_mxfp8_quantize_host(const void* x, int dtype, int64_t rows, int64_t k, int64_t row_stride,
                            uint8_t* q, uint8_t* s, int num_threads) {
  VDN_CHECK_ARG(rows >= 0 && k > 0, "rows must be nonnegative and K positive");
  VDN_CHECK_ARG(q && s && (rows == 0 || x), "null pointer");
  if (dtype != VDN_DTYPE_F32 && dtype != VDN_DTYPE_BF16 && dtype != VDN_DTYPE_F16)
    return set_error(VDN_ERR_TYPE, "expected a floating 2D weight");
  const int64_t rp = (rows + 127) / 128 * 128, kp = (k + 127) / 128 * 128;
  int nt = num_threads > 0 ? num_threads : (int)std::thread::hardware_concurrency();
  if (nt < 1) nt = 1;
  if (nt > rp / 128 + 1) nt = (int)(rp / 128 + 1);
  std::vector<std::thread> pool;
  std::vector<int> bad(nt, 0);
  const int64_t chunk = ((rp + nt - 1) / nt + 127) / 128 * 128;
  for (int t = 0; t < nt; ++t) {
    const int64_t r0 = t * chunk, r1 = std::min<int64_t>(rp, r0 + chunk);
    if (r0 >= r1) break;
    pool.emplace_back([=, &bad] { host_quantize_rows(x, dtype, r0, r1, rows, k, row_stride, kp, q, s, &bad[t]); });
  }
  for (auto& th : pool) th.join();
  for (int b : bad)
    if (b) return set_error(VDN_ERR_NONFINITE, "nonfinite MXFP8 weight");
  return VDN_OK;
}

}  // extern "C"
