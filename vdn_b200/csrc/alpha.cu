// FrameKDAAlpha on the device in two launches (reference
// src/models/linear_attention/layers.py:36-69, an fp32 island):
//   delta = frame_mean @ down^T                      [F, r]
//   u     = delta @ up^T + dt_bias                   [F, heads * d]
//   alpha = exp(-exp(A_log[head]) * softplus(u))     softplus with threshold 20
// The reference runs these as PyTorch fp32 ops (cuBLAS GEMMs, about eight
// launches, one of them a split-K GEMM on a 21-row operand); here the first
// launch spreads the F x r dot products of length `hidden` over F x r/16 CTAs
// (one warp per output, lanes striding the hidden dimension) and the second
// computes one output element per thread.
#include "common.cuh"

#include <math.h>

namespace vdn {

__global__ void __launch_bounds__(512) alpha_down_kernel(const float* __restrict__ fm, int hidden,
                                                         const float* __restrict__ down, int r,
                                                         float* __restrict__ delta) {
  const int f = blockIdx.x;
  const int j = blockIdx.y * 16 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= r) return;
  const float* x = fm + (int64_t)f * hidden;
  const float* w = down + (int64_t)j * hidden;
  float acc = 0.f;
  if ((hidden & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) == 0) {
    for (int c = lane * 4; c < hidden; c += 128) {
      const float4 a = *reinterpret_cast<const float4*>(x + c);
      const float4 b = *reinterpret_cast<const float4*>(w + c);
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
      acc = fmaf(a.z, b.z, acc);
      acc = fmaf(a.w, b.w, acc);
    }
  } else {
    for (int c = lane; c < hidden; c += 32) acc = fmaf(x[c], w[c], acc);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[(int64_t)f * r + j] = acc;
}

__global__ void __launch_bounds__(256) alpha_up_kernel(const float* __restrict__ delta, int r,
                                                       const float* __restrict__ up,
                                                       const float* __restrict__ dt_bias,
                                                       const float* __restrict__ a_log, int n_out, int d,
                                                       int F, float* __restrict__ out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= (int64_t)F * n_out) return;
  const int f = (int)(g / n_out), o = (int)(g % n_out);
  const float* dl = delta + (int64_t)f * r;
  const float* w = up + (int64_t)o * r;
  float u = 0.f;
  for (int j = 0; j < r; ++j) u = fmaf(dl[j], w[j], u);
  u += dt_bias[o];
  const float sp = u > 20.f ? u : log1pf(expf(u));
  out[g] = expf(-expf(a_log[o / d]) * sp);
}

}  // namespace vdn

using namespace vdn;

extern "C" int vdn_frame_alpha(const float* frame_mean, int F, int hidden, const float* down_w, int r,
                               const float* up_w, const float* dt_bias, const float* a_log, int heads,
                               int d, float* scratch, float* out, cudaStream_t stream) {
  VDN_CHECK_ARG(F >= 0 && hidden > 0 && r > 0 && heads > 0 && d > 0, "bad alpha extents");
  if (F == 0) return VDN_OK;
  VDN_CHECK_ARG(frame_mean && down_w && up_w && dt_bias && a_log && scratch && out, "null pointer");
  alpha_down_kernel<<<dim3(F, (r + 15) / 16), 512, 0, stream>>>(frame_mean, hidden, down_w, r, scratch);
  VDN_LAUNCH_CHECK("frame alpha (down)");
  const int n_out = heads * d;
  const int64_t total = (int64_t)F * n_out;
  alpha_up_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(scratch, r, up_w, dt_bias, a_log,
                                                                      n_out, d, F, out);
  VDN_LAUNCH_CHECK("frame alpha (up)");
  return VDN_OK;
}
