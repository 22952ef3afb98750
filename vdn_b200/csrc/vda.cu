// VDA (frame-wise bidirectional delta-rule linear attention) for sm_100a.
//
// Stage kernels, each a launch over the natural parallel unit of its stage:
//   statistics  one CTA per (frame, head): SiLU(+L2) features of k / v in
//               registers, A = sym((k*beta) k^T) fp32, B = bf16(bf16(v*beta) k^T)
//   factors     one CTA per (frame, head): in-register Gauss-Jordan inverse of
//               the SPD I + A, T = diag(alpha) inv, J = B inv
//   scan        one CTA per (head, direction, 16 state rows): rows of the state
//               evolve independently, s_t = s_{t-1} T_t + J_t, fp32
//   gather      one CTA per (frame, head, 16 rows): window complement, decayed
//   readout     one CTA per (frame, head, 256 tokens): q features, q state^T,
//               RMSNorm * w * gate, token-major bf16 store
// Reference: ec-jt/vdn src/models/linear_attention/{scan.py, delta_rule.py,
// branch.py, paper_stack.py, paper_sglang.py}.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>

namespace vdn {

constexpr int kMaxFrames = 1024;

struct FrameBounds {
  int32_t lo[kMaxFrames];
  int32_t hi[kMaxFrames];
};

// Features of one token row (d = 32 * PER lanes' worth) with the eager
// reference's bf16 rounding points (features.py:47-60): x = bf16(silu(raw));
// for q / k, norm = max(bf16(||x||), bf16(1e-6)) and x = bf16(x / norm).
template <int PER>
__device__ __forceinline__ void warp_features(const uint16_t* __restrict__ src, bool l2, float* out) {
  const int lane = threadIdx.x & 31;
  float y[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const float x = bf16_bits_to_f32(src[lane * PER + i]);
    y[i] = round_bf16(silu_f(x));
    ss += y[i] * y[i];
  }
  if (l2) {
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float nrm = fmaxf(round_bf16(sqrtf(ss)), round_bf16(1e-6f));
#pragma unroll
    for (int i = 0; i < PER; ++i) y[i] = round_bf16(__fdiv_rn(y[i], nrm));
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) out[i] = y[i];
}

// ----------------------------------------------------------------- statistics
template <int D>
__global__ void __launch_bounds__(256) stats_kernel(
    const uint16_t* __restrict__ k, int64_t k_sf, int64_t k_ss, int64_t k_sh,
    const uint16_t* __restrict__ v, int64_t v_sf, int64_t v_ss, int64_t v_sh,
    const uint16_t* __restrict__ beta, int64_t b_sf, int64_t b_ss, int64_t b_sh,
    int features_applied, int S, int H, float* __restrict__ A, float* __restrict__ B) {
  constexpr int T = D / 16;      // each thread owns a T x T tile of A and of B
  constexpr int CS = 32;         // tokens per chunk
  constexpr int PER = D / 32;    // elements per lane in a token row
  extern __shared__ float smem[];
  float* kb = smem;              // [CS][D] k * beta (fp32)
  float* kk = kb + CS * D;       // [CS][D] k features
  float* vb = kk + CS * D;       // [CS][D] bf16(v * beta)
  const int fh = blockIdx.x;
  const int f = fh / H, h = fh % H;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc_a[T][T], acc_b[T][T];
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) acc_a[i][j] = acc_b[i][j] = 0.f;

  for (int s0 = 0; s0 < S; s0 += CS) {
    __syncthreads();
    for (int t = warp; t < CS; t += 8) {
      const int s = s0 + t;
      float kf[PER], vf[PER];
      float bt = 0.f;
      if (s < S) {
        const uint16_t* kr = k + (int64_t)f * k_sf + (int64_t)s * k_ss + (int64_t)h * k_sh;
        const uint16_t* vr = v + (int64_t)f * v_sf + (int64_t)s * v_ss + (int64_t)h * v_sh;
        if (features_applied) {
#pragma unroll
          for (int i = 0; i < PER; ++i) {
            kf[i] = bf16_bits_to_f32(kr[lane * PER + i]);
            vf[i] = bf16_bits_to_f32(vr[lane * PER + i]);
          }
        } else {
          warp_features<PER>(kr, true, kf);
          warp_features<PER>(vr, false, vf);
        }
        bt = bf16_bits_to_f32(beta[(int64_t)f * b_sf + (int64_t)s * b_ss + (int64_t)h * b_sh]);
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) kf[i] = vf[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        kk[t * D + lane * PER + i] = kf[i];
        kb[t * D + lane * PER + i] = kf[i] * bt;
        vb[t * D + lane * PER + i] = round_bf16(vf[i] * bt);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int t = 0; t < CS; ++t) {
      float a[T], b[T], c[T];
#pragma unroll
      for (int i = 0; i < T; ++i) {
        a[i] = kb[t * D + ty * T + i];
        c[i] = vb[t * D + ty * T + i];
        b[i] = kk[t * D + tx * T + i];
      }
#pragma unroll
      for (int i = 0; i < T; ++i)
#pragma unroll
        for (int j = 0; j < T; ++j) {
          acc_a[i][j] = fmaf(a[i], b[j], acc_a[i][j]);
          acc_b[i][j] = fmaf(c[i], b[j], acc_b[i][j]);
        }
    }
  }
  // Symmetrise A through shared memory; round B to bf16 (reference scan.py:262-266).
  __syncthreads();
  float* as = smem;  // [D][D]
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) as[(ty * T + i) * D + tx * T + j] = acc_a[i][j];
  __syncthreads();
  float* a_out = A + (int64_t)fh * D * D;
  float* b_out = B + (int64_t)fh * D * D;
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const int r = ty * T + i, c = tx * T + j;
      a_out[r * D + c] = 0.5f * (acc_a[i][j] + as[c * D + r]);
      b_out[r * D + c] = round_bf16(acc_b[i][j]);
    }
}

// -------------------------------------------------------------------- factors
// One CTA per matrix; thread (ty, tx) holds rows {ty + 16 i} and columns
// {tx + 16 j} (i, j < D/16) of the working matrix in registers: for a fixed j
// the sixteen column groups of a warp touch sixteen consecutive words of a
// shared vector, so every shared-memory access is conflict-free.  T may alias A
// and J may alias B (each CTA reads its whole matrix before the first store),
// so those pointers are not restrict.  Non-pivoting in-place Gauss-Jordan
// inversion of the SPD M = I + A, pivots in natural order p = o + 16 jj: at
// pivot p the owners publish row p and column p through double-buffered shared
// vectors (and the pivot's owner its reciprocal, computed once), every thread
// applies the rank-1 update with one FMA per element, and the owners of row /
// column p then overwrite those entries.  J = B inv reads B rows from global
// (L2) and inv from shared memory.
// SPLIT (d = 128 only): instead of T and J, store inv = (I + A)^-1 as three bf16
// planes whose sum is the fp32 value (x = x1 + x2 + x3 exactly), each plane in the
// 128B-swizzled K-major operand layout of the tensor-core scan (two 64-column
// halves of 128 rows x 128 B per plane, 96 KB per matrix at `Tout` bytes).
template <int D, bool SPLIT = false>
__global__ void __launch_bounds__(256, 1) factor_kernel(const float* A, const float* B,
                                                        const float* __restrict__ alpha,
                                                        float* Tout, float* Jout) {
  constexpr int T = D / 16;
  extern __shared__ float smem[];
  float* rowbuf = smem;            // [2 buffers][2 rows][D]
  float* colbuf = smem + 4 * D;    // [2 buffers][2 columns][D]
  float* inv_s = smem + 8 * D;     // [D][D]
  const int64_t mat = blockIdx.x;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const float* a_in = A + mat * D * D;
  const float* b_in = B + mat * D * D;
  // Thread's T x T register tile, column pairs packed for the paired FMA (fma.rn.f32x2):
  // element (i, j) is component j & 1 of m2[i][j / 2].
  float2 m2[T][T / 2];
#define MV(i, j) ((((j) & 1) ? m2[i][(j) >> 1].y : m2[i][(j) >> 1].x))
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const int r = ty + 16 * i, c = tx + 16 * j;
      MV(i, j) = a_in[r * D + c] + (r == c ? 1.0f : 0.0f);
    }
  // Pivots are taken two at a time, p = o + 16 jj and p + 1 (o even): rows p, p + 1
  // live in row slot jj of threads ty == o, o + 1 and columns p, p + 1 in column slot
  // jj of threads tx == o, o + 1, so every slot index is a compile-time constant and
  // m stays in registers.  One step per pivot pair (64 barriers instead of 128):
  // with P the 2 x 2 pivot block, R its two rows and C its two columns,
  //   rows p, p+1    <- P^-1 R
  //   other rows     <- M - C (P^-1 R)      (a rank-2 update, two paired FMAs)
  //   columns p, p+1 <- -C P^-1,  P <- P^-1
  // which is two consecutive Gauss-Jordan pivots computed as one block step (SPD:
  // every leading 2 x 2 block of the Schur complements is SPD, so no pivoting).
#pragma unroll
  for (int jj = 0; jj < T; ++jj) {
    for (int o = 0; o < 16; o += 2) {
      const int p = o + 16 * jj;
      float* rb = rowbuf + ((o >> 1) & 1) * 2 * D;  // rows p, p + 1 of M:    rb[k * D + col]
      float* cb = colbuf + ((o >> 1) & 1) * 2 * D;  // columns p, p + 1 of M: cb[k * D + row]
      if (ty == o || ty == o + 1) {
        float* dst = rb + (ty - o) * D;
#pragma unroll
        for (int j = 0; j < T; ++j) dst[tx + 16 * j] = MV(jj, j);
      }
      if (tx == o || tx == o + 1) {
        float* dst = cb + (tx - o) * D;
#pragma unroll
        for (int i = 0; i < T; ++i) dst[ty + 16 * i] = MV(i, jj);
      }
      __syncthreads();
      const float pa = rb[p], pb = rb[p + 1], pc = rb[D + p], pd = rb[D + p + 1];
      const float rdet = __fdiv_rn(1.0f, fmaf(pa, pd, -pb * pc));
      const float i00 = pd * rdet, i01 = -pb * rdet, i10 = -pc * rdet, i11 = pa * rdet;
      float r0[T], r1[T], c0[T], c1[T];
#pragma unroll
      for (int j = 0; j < T; ++j) {
        const float x0 = rb[tx + 16 * j], x1 = rb[D + tx + 16 * j];
        r0[j] = fmaf(i00, x0, i01 * x1);
        r1[j] = fmaf(i10, x0, i11 * x1);
      }
#pragma unroll
      for (int i = 0; i < T; ++i) {
        c0[i] = cb[ty + 16 * i];
        c1[i] = cb[D + ty + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < T; ++i) {
        const float2 n0 = make_float2(-c0[i], -c0[i]), n1 = make_float2(-c1[i], -c1[i]);
#pragma unroll
        for (int jp = 0; jp < T / 2; ++jp) {
          m2[i][jp] = __ffma2_rn(n0, make_float2(r0[2 * jp], r0[2 * jp + 1]), m2[i][jp]);
          m2[i][jp] = __ffma2_rn(n1, make_float2(r1[2 * jp], r1[2 * jp + 1]), m2[i][jp]);
        }
      }
      if (ty == o || ty == o + 1) {
        const bool second = ty != o;
#pragma unroll
        for (int j = 0; j < T; ++j) MV(jj, j) = second ? r1[j] : r0[j];
      }
      if (tx == o || tx == o + 1) {
        const bool second = tx != o;
        const float q0 = second ? i01 : i00, q1 = second ? i11 : i10;  // column k of P^-1
#pragma unroll
        for (int i = 0; i < T; ++i) MV(i, jj) = -fmaf(c0[i], q0, c1[i] * q1);
        if (ty == o || ty == o + 1) MV(jj, jj) = ty == o ? q0 : q1;
      }
    }
  }
  if constexpr (SPLIT) {
    static_assert(D == 128, "split planes are laid out for d = 128");
#pragma unroll
    for (int i = 0; i < T; ++i)
#pragma unroll
      for (int j = 0; j < T; ++j) inv_s[(ty + 16 * i) * D + tx + 16 * j] = MV(i, j);
    __syncthreads();
    uint8_t* planes = reinterpret_cast<uint8_t*>(Tout) + mat * (3 * 2 * D * D);
    for (int q = threadIdx.x; q < D * (D / 8); q += blockDim.x) {
      const int r = q / (D / 8), cc = q % (D / 8), kh = cc >> 3, c = cc & 7;
      const float4 v0 = *reinterpret_cast<const float4*>(inv_s + r * D + cc * 8);
      const float4 v1 = *reinterpret_cast<const float4*>(inv_s + r * D + cc * 8 + 4);
      const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      uint32_t w[3][4];
      split3_bf16x8(x, w);
      const uint32_t off = kh * 16384 + r * 128 + ((c ^ (r & 7)) << 4);
#pragma unroll
      for (int p = 0; p < 3; ++p)
        *reinterpret_cast<uint4*>(planes + p * 32768 + off) = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
    }
    return;
  }
  const float* al = alpha ? alpha + mat * D : nullptr;
  float* t_out = Tout + mat * D * D;
  __syncthreads();  // all reads of A are done before T (which may alias A) is stored
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) {
      const int r = ty + 16 * i, c = tx + 16 * j;
      inv_s[r * D + c] = MV(i, j);
      t_out[r * D + c] = al ? al[r] * MV(i, j) : MV(i, j);
    }
  __syncthreads();
  // J = B inv
  float acc[T][T];
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) acc[i][j] = 0.f;
  for (int k4 = 0; k4 < D; k4 += 4) {
    float4 bv[T];
#pragma unroll
    for (int i = 0; i < T; ++i) bv[i] = *reinterpret_cast<const float4*>(b_in + (ty + 16 * i) * D + k4);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      float iv[T];
#pragma unroll
      for (int j = 0; j < T; ++j) iv[j] = inv_s[(k4 + kk) * D + tx + 16 * j];
#pragma unroll
      for (int i = 0; i < T; ++i) {
        const float b = kk == 0 ? bv[i].x : kk == 1 ? bv[i].y : kk == 2 ? bv[i].z : bv[i].w;
#pragma unroll
        for (int j = 0; j < T; ++j) acc[i][j] = fmaf(b, iv[j], acc[i][j]);
      }
    }
  }
  __syncthreads();  // all reads of B are done before J (which may alias B) is stored
  float* j_out = Jout + mat * D * D;
#pragma unroll
  for (int i = 0; i < T; ++i)
#pragma unroll
    for (int j = 0; j < T; ++j) j_out[(ty + 16 * i) * D + tx + 16 * j] = acc[i][j];
}
#undef MV

// ----------------------------------------------------------------------- scan
// grid (H, 2 directions, D/R row blocks); 256 threads in a 16 x 16 grid.  Rows of
// the state evolve independently, so a CTA carries R rows through all F steps;
// R (64, 32 or 16) is picked at launch so that small head counts (Ulysses
// shards) still fill the GPU.  Thread (rg, cg) owns the R/16 consecutive rows
// from rg * R/16 and the column pairs {2 cg + 32 m, 2 cg + 1 + 32 m}: for a fixed
// m the 16 column groups read one contiguous 128-byte line of T, so the shared
// memory reads are conflict-free.  T_f is double-buffered: the 64 KB bulk copy of
// T_{f+1} is issued at the start of step f and lands while step f computes.  The
// R-row state sits transposed in shared memory (k-major) and each thread
// accumulates on top of J_f with packed fp32 FMAs (fma.rn.f32x2).  Waits are
// bounded (2 s).
template <int D, int R>
__global__ void __launch_bounds__(256) scan_kernel(const float* __restrict__ Tm,
                                                   const float* __restrict__ Jm,
                                                   const float* __restrict__ seed, int F, int H,
                                                   float* __restrict__ prefix,
                                                   float* __restrict__ suffix,
                                                   int* __restrict__ status) {
  constexpr int RT = R / 16, CP = D / 32;  // rows per thread, column pairs per thread
  extern __shared__ __align__(128) float sm[];
  float* t_s = sm;                 // [2][D][D]  T_f, double buffer
  float* st_s = sm + 2 * D * D;    // [D][R]     state, transposed (k-major)
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ int abort_flag;
  const int h = blockIdx.x, dir = blockIdx.y, rb = blockIdx.z;
  const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
  const int r0 = rg * RT;
  const int row0 = rb * R + r0;
  auto frame = [&](int step) { return dir == 0 ? step : F - 1 - step; };
  auto col = [&](int m) { return 2 * cg + 32 * m; };
  auto issue = [&](int step) {
    const int64_t base = ((int64_t)frame(step) * H + h) * D * D;
    uint64_t* b = &bar[step & 1];
    sm100::mbar_arrive_expect_tx(b, D * D * 4);
    sm100::bulk_load(t_s + (step & 1) * D * D, Tm + base, D * D * 4, b);
  };
  if (tid == 0) {
    sm100::mbar_init(&bar[0], 1);
    sm100::mbar_init(&bar[1], 1);
    abort_flag = 0;
    sm100::fence_barrier_init();
  }
  for (int e = tid; e < R * D; e += 256) {
    const int rr = e / D, kk = e % D;
    st_s[kk * R + rr] = seed ? seed[((int64_t)h * D + rb * R + rr) * D + kk] : 0.f;
  }
  __syncthreads();
  if (tid == 0) issue(0);
  float* bank = dir == 0 ? prefix : suffix;
  float2 jn[RT][CP];
  {
    const int64_t base = ((int64_t)frame(0) * H + h) * D * D;
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
      for (int m = 0; m < CP; ++m)
        jn[i][m] = *reinterpret_cast<const float2*>(Jm + base + (int64_t)(row0 + i) * D + col(m));
  }
  int issued = 1;
  for (int step = 0; step < F; ++step) {
    const int64_t base = ((int64_t)frame(step) * H + h) * D * D;
    if (tid == 0 && step + 1 < F) {  // buffer (step+1)&1 was last read in step-1: all done
      issue(step + 1);
      ++issued;
    }
    float2 acc[RT][CP];
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
      for (int m = 0; m < CP; ++m) acc[i][m] = jn[i][m];
    if (step + 1 < F) {  // J of the next frame, in flight during this step
      const int64_t nb = ((int64_t)frame(step + 1) * H + h) * D * D;
#pragma unroll
      for (int i = 0; i < RT; ++i)
#pragma unroll
        for (int m = 0; m < CP; ++m)
          jn[i][m] = *reinterpret_cast<const float2*>(Jm + nb + (int64_t)(row0 + i) * D + col(m));
    }
    if (!__syncthreads_and(sm100::mbar_wait(&bar[step & 1], (step >> 1) & 1, &abort_flag))) break;
    const float* tb = t_s + (step & 1) * D * D;
#pragma unroll 4
    for (int kk = 0; kk < D; ++kk) {
      float sv[RT];
      if constexpr (RT == 4) {
        const float4 v = *reinterpret_cast<const float4*>(st_s + kk * R + r0);
        sv[0] = v.x; sv[1] = v.y; sv[2] = v.z; sv[3] = v.w;
      } else if constexpr (RT == 2) {
        const float2 v = *reinterpret_cast<const float2*>(st_s + kk * R + r0);
        sv[0] = v.x; sv[1] = v.y;
      } else {
        sv[0] = st_s[kk * R + r0];
      }
      float2 tv[CP];
#pragma unroll
      for (int m = 0; m < CP; ++m) tv[m] = *reinterpret_cast<const float2*>(tb + kk * D + col(m));
#pragma unroll
      for (int i = 0; i < RT; ++i)
#pragma unroll
        for (int m = 0; m < CP; ++m) acc[i][m] = __ffma2_rn(make_float2(sv[i], sv[i]), tv[m], acc[i][m]);
    }
    __syncthreads();  // every thread is done with T_f and the old state
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
      for (int m = 0; m < CP; ++m) {
        st_s[col(m) * R + r0 + i] = acc[i][m].x;
        st_s[(col(m) + 1) * R + r0 + i] = acc[i][m].y;
        *reinterpret_cast<float2*>(bank + base + (int64_t)(row0 + i) * D + col(m)) = acc[i][m];
      }
    __syncthreads();
  }
  if (abort_flag) {  // let every issued copy land before the CTA exits
    for (int s = 0; s < issued && s < 2; ++s) {
      const int last = issued - 1 - s;  // the newest copy on barrier last & 1
      const uint64_t t0 = sm100::globaltimer();
      while (!sm100::mbar_try_wait(&bar[last & 1], (last >> 1) & 1) &&
             sm100::globaltimer() - t0 < sm100::kWaitLimitNs) {
      }
    }
    if (tid == 0 && status) atomicExch(status, VDN_ERR_TIMEOUT);
  }
}

// --------------------------------------------------------------------- gather
template <int D, typename OutT>
__global__ void __launch_bounds__(256) gather_kernel(const float* __restrict__ prefix,
                                                     const float* __restrict__ suffix,
                                                     const float* __restrict__ alpha,
                                                     const float* __restrict__ seed, int bridge,
                                                     int F, int H, const FrameBounds bounds,
                                                     OutT* __restrict__ out, int vec) {
  constexpr int R = 16;
  __shared__ float dec_b[D], dec_a[D];
  const int t = blockIdx.x, h = blockIdx.y, rb = blockIdx.z;
  const int lo = bounds.lo[t], hi = bounds.hi[t];
  const bool has_b = lo > 0, has_a = hi + 1 < F;
  if (threadIdx.x < D) {
    const int kk = threadIdx.x;
    float pb = 1.f, pa = 1.f;
    if (bridge) {
      for (int u = max(lo, 0); u <= t; ++u) pb *= fmaxf(alpha[((int64_t)u * H + h) * D + kk], 1e-12f);
      for (int u = t; u <= min(hi, F - 1); ++u) pa *= fmaxf(alpha[((int64_t)u * H + h) * D + kk], 1e-12f);
    }
    dec_b[kk] = pb;
    dec_a[kk] = pa;
  }
  __syncthreads();
  const int64_t plane = (int64_t)D * D;
  if (vec) {
    // Eight consecutive elements per thread: 32-byte loads of each bank row, one 16-byte
    // (bf16) or 32-byte (fp32) store; every load of the thread is issued before the sums.
    for (int e = threadIdx.x * 8; e < R * D; e += blockDim.x * 8) {
      const int r = rb * R + e / D, kk = e % D;
      const int64_t off = (int64_t)r * D + kk;
      float sd[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, left[8], right[8];
      auto load8 = [](const float* src, float* dst) {
        const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
        dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
        dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
      };
      if (seed) load8(seed + h * plane + off, sd);
      if (has_b) load8(prefix + ((int64_t)(lo - 1) * H + h) * plane + off, left);
      else
        for (int i = 0; i < 8; ++i) left[i] = sd[i];
      if (has_a) load8(suffix + ((int64_t)(hi + 1) * H + h) * plane + off, right);
      else
        for (int i = 0; i < 8; ++i) right[i] = sd[i];
      float val[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) val[i] = left[i] * dec_b[kk + i] + right[i] * dec_a[kk + i];
      const int64_t o = ((int64_t)t * H + h) * plane + off;
      if constexpr (sizeof(OutT) == 2) {
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + o) = pack8(val);
      } else {
        *reinterpret_cast<float4*>(out + o) = make_float4(val[0], val[1], val[2], val[3]);
        *reinterpret_cast<float4*>(out + o + 4) = make_float4(val[4], val[5], val[6], val[7]);
      }
    }
    return;
  }
  for (int e = threadIdx.x; e < R * D; e += blockDim.x) {
    const int r = rb * R + e / D, kk = e % D;
    const int64_t off = (int64_t)r * D + kk;
    const float sd = seed ? seed[h * plane + off] : 0.f;
    const float left = has_b ? prefix[((int64_t)(lo - 1) * H + h) * plane + off] : sd;
    const float right = has_a ? suffix[((int64_t)(hi + 1) * H + h) * plane + off] : sd;
    const float val = left * dec_b[kk] + right * dec_a[kk];
    const int64_t o = ((int64_t)t * H + h) * plane + off;
    if constexpr (sizeof(OutT) == 2) reinterpret_cast<uint16_t*>(out)[o] = f32_to_bf16_bits(val);
    else out[o] = val;
  }
}

// -------------------------------------------------------------------- readout
// grid (F*H, ceil(S/256)); 256 threads = 8 warps; a warp owns 8 tokens at a time,
// lane l the output channels 4l..4l+3 (d = 128) or 2l..2l+1 (d = 64).
template <int D>
__global__ void __launch_bounds__(256) readout_kernel(
    const uint16_t* __restrict__ q, int64_t q_sf, int64_t q_ss, int64_t q_sh,
    const uint16_t* __restrict__ state, const uint16_t* __restrict__ gate, int64_t g_sf,
    int64_t g_ss, int64_t g_sh, const float* __restrict__ norm_w, float eps, int S, int H,
    uint16_t* __restrict__ out) {
  constexpr int PER = D / 32;   // channels per lane
  constexpr int TOK = 8;        // tokens per warp pass
  extern __shared__ float smem[];
  float* stT = smem;            // [D(k)][D(v)] state transposed, fp32
  float* qs = stT + D * D;      // [8 warps][D(k)][TOK]
  const int fh = blockIdx.x;
  const int f = fh / H, h = fh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint16_t* st = state + (int64_t)fh * D * D;
  for (int e = threadIdx.x; e < D * D; e += blockDim.x) {
    const int vv = e / D, kk = e % D;
    stT[kk * D + vv] = bf16_bits_to_f32(st[e]);
  }
  float w[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) w[i] = round_bf16(norm_w[lane * PER + i]);
  __syncthreads();
  float* myq = qs + warp * D * TOK;
  const int s_begin = blockIdx.y * 256;
  const int s_end = min(S, s_begin + 256);
  for (int s0 = s_begin + warp * TOK; s0 < s_end; s0 += 8 * TOK) {
    __syncwarp();
    for (int t = 0; t < TOK; ++t) {
      const int s = s0 + t;
      float qf[PER];
      if (s < s_end) {
        warp_features<PER>(q + (int64_t)f * q_sf + (int64_t)s * q_ss + (int64_t)h * q_sh, true, qf);
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) qf[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) myq[(lane * PER + i) * TOK + t] = qf[i];
    }
    __syncwarp();
    float acc[TOK][PER];
#pragma unroll
    for (int t = 0; t < TOK; ++t)
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[t][i] = 0.f;
#pragma unroll 2
    for (int kk = 0; kk < D; ++kk) {
      float sv[PER], qv[TOK];
#pragma unroll
      for (int i = 0; i < PER; ++i) sv[i] = stT[kk * D + lane * PER + i];
#pragma unroll
      for (int t = 0; t < TOK; ++t) qv[t] = myq[kk * TOK + t];
#pragma unroll
      for (int t = 0; t < TOK; ++t)
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[t][i] = fmaf(qv[t], sv[i], acc[t][i]);
    }
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
      const int s = s0 + t;
      float r[PER];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        r[i] = round_bf16(acc[t][i]);  // the readout matmul stores bf16
        ss += r[i] * r[i];
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (s >= s_end) continue;
      // Eager RMSNorm rounding points (ops/rms_norm.py:29-32): ms from the fp32
      // norm squared, bf16 reciprocal, then bf16 after each multiply.
      const float nrm = sqrtf(ss);
      const float inv = round_bf16(__fdiv_rn(1.0f, sqrtf(nrm * nrm / (float)D + eps)));
      const uint16_t* gr = gate + (int64_t)f * g_sf + (int64_t)s * g_ss + (int64_t)h * g_sh;
      uint16_t* orow = out + ((int64_t)f * S + s) * ((int64_t)H * D) + (int64_t)h * D;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int c = lane * PER + i;
        const float y = round_bf16(round_bf16(r[i] * inv) * w[i]);
        orow[c] = f32_to_bf16_bits(y * bf16_bits_to_f32(gr[c]));
      }
    }
  }
}

// Tensor-core (tcgen05) paths for d = 128, defined in vda_tc.cu.
bool tc_stats_supported(int d, const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh, const void* v,
                        int64_t v_sf, int64_t v_ss, int64_t v_sh);
int launch_stats_tc(const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sf,
                    int64_t v_ss, int64_t v_sh, const void* beta, int64_t b_sf, int64_t b_ss,
                    int64_t b_sh, int features_applied, int F, int S, int H, float* A, float* B,
                    int b_bf16, int* status, cudaStream_t stream);
bool tc_readout_supported(int d, const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh,
                          const void* state, const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh,
                          const void* out);
int launch_readout_tc(const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh, const void* state,
                      const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh, const float* norm_w,
                      float eps, int F, int S, int H, void* out, int* status, cudaStream_t stream);

static int check_d(int d) {
  if (d != 64 && d != 128) return set_error(VDN_ERR_VALUE, "head_dim must be 64 or 128, got %d", d);
  return VDN_OK;
}

template <typename K>
static int set_smem(K kernel, size_t bytes) {
  // Always raise the limit: static shared memory counts against the 48 KB default.
  VDN_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return VDN_OK;
}

static int fill_bounds(const int32_t* bounds, int F, FrameBounds* fb) {
  VDN_CHECK_ARG(bounds, "bounds must not be null");
  VDN_CHECK_ARG(F >= 1 && F <= kMaxFrames, "frames must lie in [1, %d], got %d", kMaxFrames, F);
  for (int t = 0; t < F; ++t) {
    const int lo = bounds[2 * t], hi = bounds[2 * t + 1];
    VDN_CHECK_ARG(lo <= t && t <= hi, "each inclusive window must contain its query frame");
    fb->lo[t] = lo;
    fb->hi[t] = hi;
  }
  return VDN_OK;
}

int launch_stats(const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh, const void* v,
                 int64_t v_sf, int64_t v_ss, int64_t v_sh, const void* beta, int64_t b_sf,
                 int64_t b_ss, int64_t b_sh, int features_applied, int F, int S, int H, int d,
                 float* A, float* B, cudaStream_t stream) {
  if (int rc = check_d(d)) return rc;
  VDN_CHECK_ARG(F >= 1 && S >= 1 && H >= 1, "positive F, S, H required");
  VDN_CHECK_ARG(k && v && beta && A && B, "null pointer");
  if (tc_stats_supported(d, k, k_sf, k_ss, k_sh, v, v_sf, v_ss, v_sh) && aligned32(A) && aligned32(B))
    return launch_stats_tc(k, k_sf, k_ss, k_sh, v, v_sf, v_ss, v_sh, beta, b_sf, b_ss, b_sh,
                           features_applied, F, S, H, A, B, 0, nullptr, stream);
  const size_t smem = std::max<size_t>(3 * 32 * d, (size_t)d * d) * sizeof(float);
  const auto* kp = static_cast<const uint16_t*>(k);
  const auto* vp = static_cast<const uint16_t*>(v);
  const auto* bp = static_cast<const uint16_t*>(beta);
  if (d == 128) {
    if (int rc = set_smem(stats_kernel<128>, smem)) return rc;
    stats_kernel<128><<<F * H, 256, smem, stream>>>(kp, k_sf, k_ss, k_sh, vp, v_sf, v_ss, v_sh, bp,
                                                     b_sf, b_ss, b_sh, features_applied, S, H, A, B);
  } else {
    if (int rc = set_smem(stats_kernel<64>, smem)) return rc;
    stats_kernel<64><<<F * H, 256, smem, stream>>>(kp, k_sf, k_ss, k_sh, vp, v_sf, v_ss, v_sh, bp,
                                                    b_sf, b_ss, b_sh, features_applied, S, H, A, B);
  }
  VDN_LAUNCH_CHECK("vda statistics");
  return VDN_OK;
}

int launch_factors(const float* A, const float* B, const float* alpha, int64_t n, int d, float* T,
                   float* J, cudaStream_t stream) {
  if (int rc = check_d(d)) return rc;
  VDN_CHECK_ARG(n >= 0, "n must be nonnegative");
  if (n == 0) return VDN_OK;
  VDN_CHECK_ARG(A && B && T && J, "null pointer");
  VDN_CHECK_ARG(aligned16(A) && aligned16(B), "A and B must be 16-byte aligned");
  VDN_CHECK_ARG(n < (1ll << 31), "too many matrices");
  const size_t smem = (8 * d + d * d) * sizeof(float);
  if (d == 128) {
    if (int rc = set_smem(factor_kernel<128>, smem)) return rc;
    factor_kernel<128><<<(unsigned)n, 256, smem, stream>>>(A, B, alpha, T, J);
  } else {
    if (int rc = set_smem(factor_kernel<64>, smem)) return rc;
    factor_kernel<64><<<(unsigned)n, 256, smem, stream>>>(A, B, alpha, T, J);
  }
  VDN_LAUNCH_CHECK("delta factors");
  return VDN_OK;
}

// Factor stage of the tensor-core scan: inv = (I + A)^-1 as three bf16 operand
// planes (96 KB per matrix) for each of the n matrices of A (d = 128).
int launch_factor_split(const float* A, int64_t n, void* planes, cudaStream_t stream) {
  VDN_CHECK_ARG(n >= 0 && n < (1ll << 31), "bad matrix count");
  if (n == 0) return VDN_OK;
  VDN_CHECK_ARG(A && planes && aligned16(A) && aligned16(planes), "A and planes must be 16-byte aligned");
  const size_t smem = (8 * 128 + 128 * 128) * sizeof(float);
  if (int rc = set_smem(factor_kernel<128, true>, smem)) return rc;
  factor_kernel<128, true><<<(unsigned)n, 256, smem, stream>>>(A, nullptr, nullptr, static_cast<float*>(planes),
                                                              nullptr);
  VDN_LAUNCH_CHECK("delta factors (split inverse)");
  return VDN_OK;
}

int launch_scan_tc(const void* inv_planes, const float* B, int b_bf16, const float* alpha, const float* seed,
                   int F, int H, float* prefix, float* suffix, int* status, cudaStream_t stream);

int launch_scan(const float* T, const float* J, const float* seed, int F, int H, int d,
                float* prefix, float* suffix, cudaStream_t stream) {
  if (int rc = check_d(d)) return rc;
  VDN_CHECK_ARG(F >= 1 && H >= 1, "positive F and H required");
  VDN_CHECK_ARG(T && J && prefix && suffix, "null pointer");
  VDN_CHECK_ARG(aligned16(T) && aligned16(J) && aligned16(prefix) && aligned16(suffix),
                "scan banks must be 16-byte aligned");
  int dev = 0, sms = 148;
  VDN_CUDA_TRY(cudaGetDevice(&dev));
  VDN_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  // Fewest rows per CTA (most CTAs) only when the head count leaves SMs idle.
  int R = 64;
  while (R > 16 && (int64_t)H * 2 * (d / R) < sms) R /= 2;
  const dim3 grid(H, 2, d / R);
  const size_t smem = ((size_t)2 * d * d + (size_t)d * R) * sizeof(float);
#define VDN_SCAN(DD, RR)                                                                    \
  do {                                                                                      \
    if (int rc = set_smem(scan_kernel<DD, RR>, smem)) return rc;                            \
    scan_kernel<DD, RR><<<grid, 256, smem, stream>>>(T, J, seed, F, H, prefix, suffix, nullptr); \
  } while (0)
  if (d == 128) {
    if (R == 64) VDN_SCAN(128, 64);
    else if (R == 32) VDN_SCAN(128, 32);
    else VDN_SCAN(128, 16);
  } else {
    if (R == 64) VDN_SCAN(64, 64);
    else if (R == 32) VDN_SCAN(64, 32);
    else VDN_SCAN(64, 16);
  }
#undef VDN_SCAN
  VDN_LAUNCH_CHECK("vda scan");
  return VDN_OK;
}

int launch_gather(const float* prefix, const float* suffix, const float* alpha,
                  const int32_t* bounds, const float* seed, int bridge, int F, int H, int d,
                  void* out, int out_dtype, cudaStream_t stream) {
  if (int rc = check_d(d)) return rc;
  VDN_CHECK_ARG(H >= 1, "positive H required");
  VDN_CHECK_ARG(prefix && suffix && alpha && out, "null pointer");
  FrameBounds fb;
  if (int rc = fill_bounds(bounds, F, &fb)) return rc;
  const dim3 grid(F, H, d / 16);
  const int vec = aligned16(prefix) && aligned16(suffix) && (!seed || aligned16(seed)) && aligned16(out);
  if (out_dtype == VDN_DTYPE_BF16) {
    auto* o = static_cast<__nv_bfloat16*>(out);
    if (d == 128) gather_kernel<128, __nv_bfloat16><<<grid, 256, 0, stream>>>(prefix, suffix, alpha, seed, bridge, F, H, fb, o, vec);
    else gather_kernel<64, __nv_bfloat16><<<grid, 256, 0, stream>>>(prefix, suffix, alpha, seed, bridge, F, H, fb, o, vec);
  } else if (out_dtype == VDN_DTYPE_F32) {
    auto* o = static_cast<float*>(out);
    if (d == 128) gather_kernel<128, float><<<grid, 256, 0, stream>>>(prefix, suffix, alpha, seed, bridge, F, H, fb, o, vec);
    else gather_kernel<64, float><<<grid, 256, 0, stream>>>(prefix, suffix, alpha, seed, bridge, F, H, fb, o, vec);
  } else {
    return set_error(VDN_ERR_TYPE, "out_dtype must be fp32 or bf16");
  }
  VDN_LAUNCH_CHECK("vda gather");
  return VDN_OK;
}

int launch_readout(const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh, const void* state,
                   const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh,
                   const float* norm_weight, float eps, int F, int S, int H, int d, void* out,
                   cudaStream_t stream) {
  if (int rc = check_d(d)) return rc;
  VDN_CHECK_ARG(F >= 1 && S >= 1 && H >= 1, "positive F, S, H required");
  VDN_CHECK_ARG(q && state && gate && norm_weight && out, "null pointer");
  if (tc_readout_supported(d, q, q_sf, q_ss, q_sh, state, gate, g_sf, g_ss, g_sh, out))
    return launch_readout_tc(q, q_sf, q_ss, q_sh, state, gate, g_sf, g_ss, g_sh, norm_weight, eps, F, S,
                             H, out, nullptr, stream);
  const size_t smem = ((size_t)d * d + 8 * d * 8) * sizeof(float);
  const dim3 grid(F * H, (S + 255) / 256);
  const auto* qp = static_cast<const uint16_t*>(q);
  const auto* sp = static_cast<const uint16_t*>(state);
  const auto* gp = static_cast<const uint16_t*>(gate);
  auto* op = static_cast<uint16_t*>(out);
  if (d == 128) {
    if (int rc = set_smem(readout_kernel<128>, smem)) return rc;
    readout_kernel<128><<<grid, 256, smem, stream>>>(qp, q_sf, q_ss, q_sh, sp, gp, g_sf, g_ss, g_sh,
                                                      norm_weight, eps, S, H, op);
  } else {
    if (int rc = set_smem(readout_kernel<64>, smem)) return rc;
    readout_kernel<64><<<grid, 256, smem, stream>>>(qp, q_sf, q_ss, q_sh, sp, gp, g_sf, g_ss, g_sh,
                                                     norm_weight, eps, S, H, op);
  }
  VDN_LAUNCH_CHECK("vda readout");
  return VDN_OK;
}

}  // namespace vdn

using namespace vdn;

extern "C" {

int vdn_delta_factors(const float* A, const float* B, const float* alpha, int64_t n, int d,
                      float* T, float* J, cudaStream_t stream) {
  return launch_factors(A, B, alpha, n, d, T, J, stream);
}

int vdn_vda_statistics(const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh, const void* v,
                       int64_t v_sf, int64_t v_ss, int64_t v_sh, const void* beta, int64_t b_sf,
                       int64_t b_ss, int64_t b_sh, int features_applied, int F, int S, int H,
                       int d, float* A, float* B, cudaStream_t stream) {
  return launch_stats(k, k_sf, k_ss, k_sh, v, v_sf, v_ss, v_sh, beta, b_sf, b_ss, b_sh,
                      features_applied, F, S, H, d, A, B, stream);
}

int vdn_vda_scan(const float* T, const float* J, const float* seed, int F, int H, int d,
                 float* prefix, float* suffix, cudaStream_t stream) {
  return launch_scan(T, J, seed, F, H, d, prefix, suffix, stream);
}

int vdn_vda_gather(const float* prefix, const float* suffix, const float* alpha,
                   const int32_t* bounds, const float* seed, int bridge, int F, int H, int d,
                   void* out, int out_dtype, cudaStream_t stream) {
  return launch_gather(prefix, suffix, alpha, bounds, seed, bridge, F, H, d, out, out_dtype, stream);
}

int vdn_vda_readout(const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh, const void* state,
                    const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh,
                    const float* norm_weight, float eps, int F, int S, int H, int d, void* out,
                    cudaStream_t stream) {
  return launch_readout(q, q_sf, q_ss, q_sh, state, gate, g_sf, g_ss, g_sh, norm_weight, eps, F,
                        S, H, d, out, stream);
}

// Workspace regions of vdn_vda_forward, each 256-byte aligned.  d = 128 (tensor-core
// scan): A, then the forward bank over it (A is dead once the factors have read it),
// B, the split inverses (three bf16 planes), the reverse bank, the gathered state
// (bf16): 20 bytes per state element.  d = 64: A/T and B/J (the factors overwrite the
// statistics), prefix, suffix, state: 18 bytes per state element.
struct VdaWorkspace {
  float* A;
  float* B;
  void* planes;
  float* prefix;
  float* suffix;
  void* state;
  size_t bytes;
};

static VdaWorkspace vda_workspace(void* base, int F, int H, int d) {
  const size_t plane = (size_t)F * H * d * d;
  auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  char* ws = static_cast<char*>(base);
  VdaWorkspace w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = ws ? ws + off : nullptr;
    off += up(bytes);
    return p;
  };
  if (d == 128) {
    w.A = reinterpret_cast<float*>(take(plane * 4));
    w.prefix = w.A;
    w.B = reinterpret_cast<float*>(take(plane * 4));
    w.planes = take(plane * 6);
    w.suffix = reinterpret_cast<float*>(take(plane * 4));
  } else {
    w.A = reinterpret_cast<float*>(take(plane * 4));
    w.B = reinterpret_cast<float*>(take(plane * 4));
    w.prefix = reinterpret_cast<float*>(take(plane * 4));
    w.suffix = reinterpret_cast<float*>(take(plane * 4));
  }
  w.state = take(plane * 2);
  w.bytes = off;
  return w;
}

int vdn_vda_factor_inverse(const float* A, int64_t n, void* planes, cudaStream_t stream) {
  return launch_factor_split(A, n, planes, stream);
}

int vdn_vda_scan_tc(const void* planes, const float* B, const float* alpha, const float* seed, int F, int H,
                    float* prefix, float* suffix, int* status, cudaStream_t stream) {
  return launch_scan_tc(planes, B, 0, alpha, seed, F, H, prefix, suffix, status, stream);
}

int vdn_vda_scan_tc_bf16(const void* planes, const void* B, const float* alpha, const float* seed, int F,
                         int H, float* prefix, float* suffix, int* status, cudaStream_t stream) {
  return launch_scan_tc(planes, static_cast<const float*>(B), 1, alpha, seed, F, H, prefix, suffix, status,
                        stream);
}

size_t vdn_vda_workspace_size(int F, int S, int H, int d) {
  (void)S;
  return vda_workspace(nullptr, F, H, d).bytes;
}

int vdn_vda_forward(const void* q, const void* k, const void* v, int64_t qkv_ss, int64_t qkv_sh,
                    const void* beta, int64_t b_ss, int64_t b_sh, const void* gate, int64_t g_ss,
                    int64_t g_sh, const float* alpha, const float* norm_weight, float eps,
                    const int32_t* bounds, const float* seed, int bridge, int F, int S, int H,
                    int d, void* out, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream) {
  if (int rc = check_d(d)) return rc;
  VDN_CHECK_ARG(F >= 1 && S >= 1 && H >= 1, "positive F, S, H required");
  VDN_CHECK_ARG(q && k && v && beta && gate && alpha && norm_weight && out, "null pointer");
  const size_t need = vdn_vda_workspace_size(F, S, H, d);
  VDN_CHECK_ARG(workspace && workspace_bytes >= need, "workspace too small: need %zu bytes", need);
  VDN_CHECK_ARG(aligned32(workspace), "workspace must be 32-byte aligned");
  FrameBounds fb;
  if (int rc = fill_bounds(bounds, F, &fb)) return rc;
  const VdaWorkspace w = vda_workspace(workspace, F, H, d);
  float *A = w.A, *B = w.B, *prefix = w.prefix, *suffix = w.suffix;
  void* state = w.state;
  const int64_t sf = (int64_t)S * qkv_ss;
  // d = 128 with the tensor-core statistics: B leaves the statistics in bf16 (its values
  // are bf16 either way) and reaches the scan by TMA.
  const int b_bf16 = d == 128 && tc_stats_supported(d, k, sf, qkv_ss, qkv_sh, v, sf, qkv_ss, qkv_sh);
  if (b_bf16) {
    if (int rc = launch_stats_tc(k, sf, qkv_ss, qkv_sh, v, sf, qkv_ss, qkv_sh, beta, (int64_t)S * b_ss, b_ss, b_sh,
                                 0, F, S, H, A, B, 1, nullptr, stream))
      return rc;
  } else if (int rc = launch_stats(k, sf, qkv_ss, qkv_sh, v, sf, qkv_ss, qkv_sh, beta, (int64_t)S * b_ss,
                                   b_ss, b_sh, 0, F, S, H, d, A, B, stream)) {
    return rc;
  }
  if (d == 128) {  // inverse only, then the tensor-core scan folds alpha and B into each step
    VDN_CHECK_ARG(aligned16(alpha) && (!seed || aligned16(seed)), "alpha and seed must be 16-byte aligned");
    if (int rc = launch_factor_split(A, (int64_t)F * H, w.planes, stream)) return rc;
    if (int rc = launch_scan_tc(w.planes, B, b_bf16, alpha, seed, F, H, prefix, suffix, nullptr, stream))
      return rc;
  } else {
    if (int rc = launch_factors(A, B, alpha, (int64_t)F * H, d, A, B, stream)) return rc;
    if (int rc = launch_scan(A, B, seed, F, H, d, prefix, suffix, stream)) return rc;
  }
  if (int rc = launch_gather(prefix, suffix, alpha, bounds, seed, bridge, F, H, d, state,
                             VDN_DTYPE_BF16, stream))
    return rc;
  return launch_readout(q, sf, qkv_ss, qkv_sh, state, gate, (int64_t)S * g_ss, g_ss, g_sh,
                        norm_weight, eps, F, S, H, d, out, stream);
}

}  // extern "C"
