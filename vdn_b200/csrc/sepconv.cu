// The linear branch's separable short conv on the device (reference
// src/models/linear_attention/features.py:133-209 LinearAttentionSepConv and
// :12-40 the temporal shift): a depthwise 5x5 SPATIAL conv per frame, then a
// depthwise 5-tap TEMPORAL conv across frames, both bias-free with zero padding.
// Output is the conv result in bf16; the branch's SiLU [-> L2Norm] features are
// applied afterwards by the statistics / readout kernels, as for unconvolved
// projections.
//
// Rounding points follow the reference: the spatial half is a bf16 tensor (fp32
// accumulation of the 25 exact bf16 products, one rounding); the temporal half
// sums its five exact products in fp32, taps in order, and rounds once (the
// fused form of the reference's compiled CUDA path; the eager CPU shift rounds
// every product and partial sum and differs by at most a bf16 ulp or two).
//
// Layout: tokens are rows of C = heads * head_dim contiguous channels (any row
// stride), frame-major, row-major (y, x) inside a frame.  Thread = (token, 8
// channels); weights are tap-major ([taps, C]) so a thread's 8 channels of one
// tap are one 16-byte load.
#include "common.cuh"

namespace vdn {

__global__ void __launch_bounds__(256) sepconv_spatial_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                              int F, int gh, int gw, int C,
                                                              const uint16_t* __restrict__ w,
                                                              uint16_t* __restrict__ out) {
  const int groups = C >> 3;
  const int S = gh * gw;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)F * S * groups) return;
  const int64_t token = g / groups;
  const int cg = (int)(g - token * groups);
  const int t = (int)(token / S), p = (int)(token - (int64_t)t * S);
  const int y = p / gw, xx = p - y * gw;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int dy = 0; dy < 5; ++dy) {
    const int yy = y + dy - 2;
    if (yy < 0 || yy >= gh) continue;
#pragma unroll
    for (int dx = 0; dx < 5; ++dx) {
      const int xc = xx + dx - 2;
      if (xc < 0 || xc >= gw) continue;
      const int64_t src = (int64_t)t * S + (int64_t)yy * gw + xc;
      float xv[8], wv[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(x + src * ldx) + cg), xv);
      unpack8(__ldg(reinterpret_cast<const uint4*>(w + (int64_t)(dy * 5 + dx) * C) + cg), wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(xv[i], wv[i], acc[i]);
    }
  }
  reinterpret_cast<uint4*>(out + token * C)[cg] = pack8(acc);
}

__global__ void __launch_bounds__(256) sepconv_temporal_kernel(const uint16_t* __restrict__ s, int F, int S,
                                                               int C, const uint16_t* __restrict__ w,
                                                               uint16_t* __restrict__ out, int64_t ldo) {
  const int groups = C >> 3;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)F * S * groups) return;
  const int64_t token = g / groups;
  const int cg = (int)(g - token * groups);
  const int t = (int)(token / S), p = (int)(token - (int64_t)t * S);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
  for (int dt = 0; dt < 5; ++dt) {
    const int tt = t + dt - 2;
    if (tt < 0 || tt >= F) continue;  // zero padding: the tap contributes an exact 0
    float sv[8], wv[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(s + ((int64_t)tt * S + p) * C) + cg), sv);
    unpack8(__ldg(reinterpret_cast<const uint4*>(w + (int64_t)dt * C) + cg), wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(sv[i], wv[i]));
  }
  reinterpret_cast<uint4*>(out + token * ldo)[cg] = pack8(acc);
}

}  // namespace vdn

using namespace vdn;

extern "C" int vdn_sepconv(const void* x, int64_t x_ld, int F, int gh, int gw, int C, const void* w_spatial,
                           const void* w_temporal, void* scratch, void* out, int64_t out_ld,
                           cudaStream_t stream) {
  VDN_CHECK_ARG(F >= 0 && gh > 0 && gw > 0 && C > 0 && C % 8 == 0, "bad short-conv extents (C % 8 == 0)");
  if (F == 0) return VDN_OK;
  VDN_CHECK_ARG(x && w_spatial && w_temporal && scratch && out, "null pointer");
  VDN_CHECK_ARG(aligned16(x) && aligned16(w_spatial) && aligned16(w_temporal) && aligned16(scratch) &&
                    aligned16(out) && x_ld % 8 == 0 && out_ld % 8 == 0 && x_ld >= C && out_ld >= C,
                "short-conv operands must be 16-byte aligned with row strides % 8 == 0 and >= C");
  const int64_t threads = (int64_t)F * gh * gw * (C / 8);
  const unsigned grid = (unsigned)((threads + 255) / 256);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  uint16_t* sp = static_cast<uint16_t*>(scratch);
  sepconv_spatial_kernel<<<grid, 256, 0, stream>>>(xp, x_ld, F, gh, gw, C,
                                                   static_cast<const uint16_t*>(w_spatial), sp);
  VDN_LAUNCH_CHECK("short conv (spatial)");
  sepconv_temporal_kernel<<<grid, 256, 0, stream>>>(sp, F, gh * gw, C, static_cast<const uint16_t*>(w_temporal),
                                                    static_cast<uint16_t*>(out), out_ld);
  VDN_LAUNCH_CHECK("short conv (temporal)");
  return VDN_OK;
}
