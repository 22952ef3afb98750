// Window-softmax combine for the hybrid block, sm_100a.
//
// The frame window [t-r, t+r] is computed as 2r+1 dense attentions (query frame
// t against key frame t+delta, one batched library call per delta: no key/value
// duplication).  This kernel merges the partial outputs by their log-sum-exps
// (out = sum_j exp(lse_j - m) o_j / sum_j exp(lse_j - m)), rounds to bf16,
// applies the per-(token, head) softmax gate (bf16), and writes either bf16
// (the Ulysses return buffer) and/or MXFP8 codes + swizzled E8M0 scales that
// the output-projection GEMM consumes directly -- the gated softmax output is
// never materialised in bf16 on the single-GPU path.
// One thread per 32-element block of the [T, H*d] output; lanes 4i..4i+3 pack
// their scale bytes into one 32-bit store, as in the quantiser.  Capped at 64
// registers (four CTAs, 32 warps per SM): with 90 registers two CTAs fit and the
// loads in flight fell short of HBM (config 3: 0.232 -> 0.160 ms).
// Reference: window_softmax_reference / decomposed window softmax and
// apply_softmax_gate (ec-jt/vdn src/models/softmax_attention/window.py:56-111,
// decomposed.py, hybrid_attention.py:217-222).
#include "common.cuh"

namespace vdn {

constexpr int kMaxPartials = 5;

struct Partials {
  const uint16_t* out[kMaxPartials];   // [rows_j, H*d] bf16, token-major
  const float* lse[kMaxPartials];      // [batches_j, H, S] fp32
  int batch0[kMaxPartials];            // batch index = frame - batch0
  int frame_lo[kMaxPartials];          // valid query frames [frame_lo, frame_hi]
  int frame_hi[kMaxPartials];
  int n;
};

__device__ __forceinline__ uint16_t e4m3x2_w(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(256, 4) window_merge_kernel(
    const Partials P, int F, int S, int H, int d, const uint16_t* __restrict__ gate, int64_t g_ss,
    int64_t g_sh, uint16_t* __restrict__ out, int64_t out_ld, int64_t out_hs, uint8_t* __restrict__ q,
    uint8_t* __restrict__ s, int64_t rows_pad) {
  const int64_t K = (int64_t)H * d;
  const int64_t nblk = K >> 5;
  const int64_t T = (int64_t)F * S;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (q ? rows_pad : T) * nblk;
  const bool active = g < total;
  const int64_t r = active ? g / nblk : 0;
  const int64_t c = active ? g - r * nblk : 0;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = 0.f;
  if (active && r < T) {
    const int f = (int)(r / S), sidx = (int)(r - (int64_t)f * S);
    const int h = (int)((c * 32) / d);
    float lse[kMaxPartials];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxPartials; ++j) {
      lse[j] = -INFINITY;
      if (j < P.n && f >= P.frame_lo[j] && f <= P.frame_hi[j]) {
        const int b = f - P.batch0[j];
        lse[j] = P.lse[j][((int64_t)b * H + h) * S + sidx];
        m = fmaxf(m, lse[j]);
      }
    }
    float wsum = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPartials; ++j) {
      if (lse[j] == -INFINITY) continue;
      const float w = __expf(lse[j] - m);
      wsum += w;
      const int b = f - P.batch0[j];
      const uint4* src = reinterpret_cast<const uint4*>(P.out[j] + ((int64_t)b * S + sidx) * K + c * 32);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float x[8];
        unpack8(__ldg(src + k), x);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[8 * k + e] = fmaf(w, x[e], v[8 * k + e]);
      }
    }
    const float inv = wsum > 0.f ? 1.0f / wsum : 0.f;
    const float gt = bf16_bits_to_f32(gate[r * g_ss + (int64_t)h * g_sh]);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float a = v[i] * inv, b2 = v[i + 1] * inv;
      round_bf16_pair(a, b2);
      a *= gt;
      b2 *= gt;
      round_bf16_pair(a, b2);
      v[i] = a;
      v[i + 1] = b2;
    }
    if (out) {
      uint4* dst = reinterpret_cast<uint4*>(out + r * out_ld + (int64_t)h * out_hs + (c * 32) % d);
#pragma unroll
      for (int k = 0; k < 4; ++k) dst[k] = pack_exact8(v + 8 * k);
    }
  }
  if (!q) return;
  // MXFP8 of the bf16 block (same rule as the quantiser; padding rows are zero).
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint32_t b = __float_as_uint(v[i]) & 0x7FFFFFFFu;
    amax_bits = b > amax_bits ? b : amax_bits;
  }
  const int biased = (int)((amax_bits >> 23) & 255u);
  int e = biased - 135 + (amax_bits > (((uint32_t)biased << 23) | 0x600000u) ? 1 : 0);
  if (e < -127) e = -127;
  const float sc = __uint_as_float((uint32_t)(127 - e) << 23);
  const unsigned lane = threadIdx.x & 31;
  uint32_t word = (uint32_t)(e + 127) << (8 * (lane & 3));
  word |= __shfl_xor_sync(0xffffffffu, word, 1);
  word |= __shfl_xor_sync(0xffffffffu, word, 2);
  if (!active) return;
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    packed[i] = (uint32_t)e4m3x2_w(v[4 * i + 1] * sc, v[4 * i] * sc) |
                ((uint32_t)e4m3x2_w(v[4 * i + 3] * sc, v[4 * i + 2] * sc) << 16);
  uint4* qp = reinterpret_cast<uint4*>(q + r * K + c * 32);
  qp[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  qp[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  if ((lane & 3) == 0) {
    const int64_t off = ((r >> 7) * (K >> 7) + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4;
    *reinterpret_cast<uint32_t*>(s + off) = word;
  }
}

}  // namespace vdn

using namespace vdn;

extern "C" int vdn_window_merge(int n_partials, const void* const* outs, const float* const* lses,
                                const int* batch0, const int* frame_lo, const int* frame_hi, int F,
                                int S, int H, int d, const void* gate, int64_t g_ss, int64_t g_sh,
                                void* out_bf16, int64_t out_ld, int64_t out_hs, uint8_t* q,
                                uint8_t* s, cudaStream_t stream) {
  VDN_CHECK_ARG(n_partials >= 1 && n_partials <= kMaxPartials, "1..%d partials supported", kMaxPartials);
  VDN_CHECK_ARG(F >= 1 && S >= 1 && H >= 1 && d >= 32 && d % 32 == 0, "bad window geometry");
  VDN_CHECK_ARG(outs && lses && batch0 && frame_lo && frame_hi && gate, "null pointer");
  VDN_CHECK_ARG(out_bf16 || (q && s), "nothing to write: give out_bf16 and/or q + s");
  const int64_t K = (int64_t)H * d;
  VDN_CHECK_ARG(!q || K % 128 == 0, "MXFP8 output needs H*d to be a multiple of 128");
  VDN_CHECK_ARG(!out_bf16 || (out_hs >= d && out_hs % 8 == 0 && out_ld >= (int64_t)H * out_hs &&
                               out_ld % 8 == 0 && aligned16(out_bf16)),
                "out_bf16 needs 16-byte aligned head / row strides with out_hs >= d, out_ld >= H*out_hs");
  Partials P{};
  P.n = n_partials;
  for (int j = 0; j < n_partials; ++j) {
    VDN_CHECK_ARG(outs[j] && lses[j] && aligned16(outs[j]), "partial %d: null or misaligned", j);
    VDN_CHECK_ARG(frame_lo[j] >= 0 && frame_hi[j] < F && frame_lo[j] - batch0[j] >= 0,
                  "partial %d: bad frame range", j);
    P.out[j] = static_cast<const uint16_t*>(outs[j]);
    P.lse[j] = lses[j];
    P.batch0[j] = batch0[j];
    P.frame_lo[j] = frame_lo[j];
    P.frame_hi[j] = frame_hi[j];
  }
  const int64_t T = (int64_t)F * S;
  const int64_t rows_pad = (T + 127) / 128 * 128;
  const int64_t threads = (q ? rows_pad : T) * (K / 32);
  window_merge_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
      P, F, S, H, d, static_cast<const uint16_t*>(gate), g_ss, g_sh, static_cast<uint16_t*>(out_bf16),
      out_ld, out_hs, q, s, rows_pad);
  VDN_LAUNCH_CHECK("window merge");
  return VDN_OK;
}
