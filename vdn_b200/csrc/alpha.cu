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

// ----------------------------------------------------------------- frame sums
// Per-frame fp32 column sums of bf16 rows, the input of FrameKDAAlpha (the
// reference's frame mean, branch.py:450-452, and the sequence-parallel frame sums,
// ulysses_runtime.py:606-635): out[f, c] = (sum of x[r, c] over rows r in
// [bounds[f], bounds[f + 1])) / divisor.  grid (width / 256, frames), 256 threads =
// 32 column lanes (8 columns each: one 16-byte load per row, a warp reads 512
// contiguous bytes) x 8 row groups (rows g, g + 8, ...; four rows in flight per
// thread).  The row groups are added in a fixed order, so the sums are the same on
// every run (the reference replaced an atomic reduction for that reason).
constexpr int kFrameSumsMax = 1024;
struct FrameRows {
  int32_t b[kFrameSumsMax + 1];
};

__global__ void __launch_bounds__(256) frame_sums_kernel(const uint16_t* __restrict__ x, int64_t ld,
                                                         int64_t width, const __grid_constant__ FrameRows fr,
                                                         float divisor, float* __restrict__ out) {
  __shared__ __align__(16) float part[8][256];
  const int f = blockIdx.y;
  const int lc = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * 256;
  const int64_t col = c0 + lc * 8;
  const int r1 = fr.b[f + 1];
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto add = [&](const uint4& v) {
    float e[8];
    unpack8(v, e);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] += e[k];
  };
  if (col < width) {
    const uint16_t* px = x + col;
    int r = fr.b[f] + g;
    for (; r + 24 < r1; r += 32) {
      const uint4 v0 = __ldg(reinterpret_cast<const uint4*>(px + (int64_t)r * ld));
      const uint4 v1 = __ldg(reinterpret_cast<const uint4*>(px + (int64_t)(r + 8) * ld));
      const uint4 v2 = __ldg(reinterpret_cast<const uint4*>(px + (int64_t)(r + 16) * ld));
      const uint4 v3 = __ldg(reinterpret_cast<const uint4*>(px + (int64_t)(r + 24) * ld));
      add(v0);
      add(v1);
      add(v2);
      add(v3);
    }
    for (; r < r1; r += 8) add(__ldg(reinterpret_cast<const uint4*>(px + (int64_t)r * ld)));
  }
  float4* dst = reinterpret_cast<float4*>(&part[g][lc * 8]);
  dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  __syncthreads();
  const int64_t c = c0 + threadIdx.x;
  if (c < width) {
    float s = part[0][threadIdx.x];
#pragma unroll
    for (int k = 1; k < 8; ++k) s += part[k][threadIdx.x];
    out[(int64_t)f * width + c] = __fdiv_rn(s, divisor);
  }
}

}  // namespace vdn

using namespace vdn;

extern "C" int vdn_frame_sums(const void* x, int64_t ld, int64_t rows, int64_t width, const int32_t* bounds,
                              int frames, float divisor, float* out, cudaStream_t stream) {
  VDN_CHECK_ARG(frames >= 1 && frames <= kFrameSumsMax, "frames must lie in [1, %d]", kFrameSumsMax);
  VDN_CHECK_ARG(rows >= 0 && rows < (1ll << 31) && width > 0, "bad extents");
  VDN_CHECK_ARG(bounds && out && (x || rows == 0), "null pointer");
  VDN_CHECK_ARG(width % 8 == 0 && ld % 8 == 0 && ld >= width && aligned16(x),
                "x must be 16-byte aligned with width and row stride multiples of 8 elements");
  VDN_CHECK_ARG(divisor != 0.0f, "divisor must be nonzero");
  FrameRows fr;
  for (int f = 0; f <= frames; ++f) {
    VDN_CHECK_ARG(bounds[f] >= 0 && bounds[f] <= rows && (f == 0 || bounds[f] >= bounds[f - 1]),
                  "bounds must be nondecreasing row offsets within [0, rows]");
    fr.b[f] = bounds[f];
  }
  frame_sums_kernel<<<dim3((unsigned)((width + 255) / 256), (unsigned)frames), 256, 0, stream>>>(
      static_cast<const uint16_t*>(x), ld, width, fr, divisor, out);
  VDN_LAUNCH_CHECK("frame sums");
  return VDN_OK;
}

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
