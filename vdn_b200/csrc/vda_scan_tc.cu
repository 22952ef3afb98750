// Bidirectional VDA scan on sm_100a tensor cores (d = 128).
//
// One CTA per (head, direction) carries the whole fp32 state through the F frames:
//     P_f = (P_{f-1} diag(alpha_f) + B_f) (I + A_f)^-1
// which is the reference recurrence s_t = s_{t-1} T_t + J_t with T = diag(alpha) inv
// and J = B inv (scan.py:176-261, delta_rule.py:45-60) with the injection folded into
// the step, so the factor stage only inverts.  Each step's product runs on tcgen05
// (kind::f16, fp32 accumulator in TMEM) with both operands split into three bf16
// parts (x = x1 + x2 + x3 exactly): the six products x_i inv_j with i + j <= 4 give
// the fp32 result to within 2^-27 of each term, the accuracy of an fp32 GEMM.
//
// Roles (576 threads):
//   warp 0 lane 0   bulk-copies the next frame's split inverse (96 KB, written in
//                   the operand layout by the factor kernel) into shared memory
//   warp 1          TMEM allocation; lane 0 issues the 48 MMAs of a step (each
//                   64-deep K half into its own 128 columns)
//   warps 2-17      a quarter row of the state per thread (thread = TMEM lane x 32
//                   columns): read P_{f-1} from TMEM, form X_f = P_{f-1} alpha_f + B_f
//                   and write its three bf16 parts into the A operand (128B-swizzled,
//                   K-major); then, while the tensor cores compute P_f, store P_{f-1}
//                   to its bank (whole 128-byte lines after an in-warp transpose)
// The copy of inverse f+1 lands while the rows of step f are formed.  With B in bf16
// (the forward: the statistics round B to bf16 anyway) B_f arrives by TMA as a
// 128B-swizzled 32 KB tile, and alpha_f (512 bytes) by a bulk copy on the same
// barrier, while the previous product runs; the fp32-B form reads B row by row, and
// alpha from global memory or (up to 64 frames) a copy staged at the start.  A step is the
// product (48 MMAs, ~3.2k cycles) plus the rows' TMEM read and X formation; the bank
// stores, issued after X, overlap the product.  Every wait
// is bounded (2 s); a timeout aborts all roles, lets copies and MMAs in flight
// finish, frees TMEM and reports VDN_ERR_TIMEOUT through `status`.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cstring>

namespace vdn {
namespace vscan {

using namespace sm100;

constexpr int D = 128;
constexpr int PLANE = D * D * 2;            // one bf16 part: 2 x (128 rows x 128 B) = 32 KB
constexpr int OPER = 3 * PLANE;             // three parts = 96 KB
constexpr int ROW_WARPS = 16;               // four warps per TMEM lane quadrant (column quarters)
constexpr int THREADS = 64 + 32 * ROW_WARPS;  // warp 0 producer, warp 1 MMA, warps 2-17 rows
constexpr int ALPHA_FRAMES = 64;            // alpha of up to this many frames staged in shared memory
constexpr size_t SMEM = 1024 + 2 * OPER + ALPHA_FRAMES * D * 4 + 256;
constexpr int BTILE = D * D * 2;            // bf16 B_f: two 64-column halves of 128 rows x 128 B
constexpr size_t SMEM_BH = 1024 + 2 * OPER + BTILE + D * 4 + 256;  // + alpha_f, staged with B_f
static_assert(SMEM <= 232448 && SMEM_BH <= 232448, "shared memory per CTA");

struct Params {
  const uint8_t* inv;      // [F, H] split inverses, OPER bytes each
  const float* B;          // [F, H, d, d] fp32 (B of the statistics); unused on the bf16 path
  const float* alpha;      // [F, H, d] fp32
  const float* seed;       // [H, d, d] or null
  float* prefix;           // [F, H, d, d] forward states
  float* suffix;           // [F, H, d, d] reverse states
  int F, H;
  int* status;
};

// Byte offset of 16-byte chunk `c` (0..15 along K) of row `r` in a K-major
// 128B-swizzled part (two 64-column halves of 16 KB).
__device__ __forceinline__ uint32_t oper_off(uint32_t r, uint32_t c) {
  return (c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// BH: B_f in bf16 through a tensor map (tb: [F*H*128 rows, 128 cols], 64 x 128 boxes,
// 128B swizzle), staged in shared memory by TMA.
template <bool BH>
__global__ void __launch_bounds__(THREADS, 1) scan_tc_kernel(const __grid_constant__ CUtensorMap tb,
                                                             const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;                        // A operand: X_f parts
  uint8_t* sI = smem + OPER;                 // B operand: inv_f parts
  uint8_t* sB = smem + 2 * OPER;             // BH: B_f tile
  float* sAlpha = reinterpret_cast<float*>(smem + 2 * OPER);   // !BH: [F][D] when F <= ALPHA_FRAMES
  float* sAl = reinterpret_cast<float*>(smem + 2 * OPER + BTILE);  // BH: alpha_f
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * OPER + (BH ? BTILE + D * 4 : ALPHA_FRAMES * D * 4));
  uint64_t* inv_full = bars;
  uint64_t* inv_empty = bars + 1;
  uint64_t* x_ready = bars + 2;
  uint64_t* acc_full = bars + 3;
  uint64_t* mma_drain = bars + 4;
  uint64_t* b_full = bars + 5;
  uint64_t* b_empty = bars + 6;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x >> 1, dir = blockIdx.x & 1;
  const int F = p.F, H = p.H;
  auto frame = [&](int step) { return dir == 0 ? step : F - 1 - step; };

  if (tid == 0) {
    mbar_init(inv_full, 1);
    mbar_init(inv_empty, 1);
    mbar_init(x_ready, ROW_WARPS);  // one arrival per row warp
    mbar_init(acc_full, 1);
    mbar_init(mma_drain, 1);
    mbar_init(b_full, 1);
    mbar_init(b_empty, ROW_WARPS);  // one arrival per row warp once it has read B_f
    *abort_flag = 0;
    fence_barrier_init();
    if (BH) prefetch_tensormap(&tb);
  }
  const bool alpha_smem = !BH && F <= ALPHA_FRAMES;
  if (alpha_smem)
    for (int i = tid; i < F * D / 4; i += THREADS)
      reinterpret_cast<float4*>(sAlpha)[i] =
          __ldg(reinterpret_cast<const float4*>(p.alpha + ((int64_t)(i / (D / 4)) * H + h) * D) + i % (D / 4));
  if (warp == 1) tmem_alloc(tmem_holder, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int issued = 0, b_issued = 0;
      for (int step = 0; step < F && !*abort_flag; ++step) {
        if (BH) {  // B_f and alpha_f once the rows have formed X_{f-1} (while the previous product runs)
          if (!mbar_wait(b_empty, (step & 1) ^ 1, abort_flag)) break;
          mbar_arrive_expect_tx(b_full, BTILE + D * 4);
          const int brow = (frame(step) * H + h) * D;
          tma_load_2d(sB, &tb, b_full, 0, brow);
          tma_load_2d(sB + BTILE / 2, &tb, b_full, 64, brow);
          bulk_load(sAl, p.alpha + ((int64_t)frame(step) * H + h) * D, D * 4, b_full);
          ++b_issued;
        }
        if (!mbar_wait(inv_empty, (step & 1) ^ 1, abort_flag)) break;
        const uint8_t* src = p.inv + ((int64_t)frame(step) * H + h) * OPER;
        mbar_arrive_expect_tx(inv_full, OPER);
#pragma unroll
        for (int part = 0; part < 3; ++part) bulk_load(sI + part * PLANE, src + part * PLANE, PLANE, inv_full);
        // The next frame's inverse moves into L2 during this step, so its copy into
        // shared memory (which has to wait for this step's MMAs) reads from L2.
        if (step + 1 < F) bulk_prefetch_l2(p.inv + ((int64_t)frame(step + 1) * H + h) * OPER, OPER);
        ++issued;
      }
      if (*abort_flag && issued) {  // the last copy must land before the CTA may exit
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(inv_full, (issued - 1) & 1) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
      if (*abort_flag && b_issued) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(b_full, (b_issued - 1) & 1) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------------------- MMA
      constexpr uint32_t kIdesc = idesc_bf16(128, 128, 0, 0);
      // Split products x_i inv_j kept: i + j <= 4 (parts counted from 1), smallest
      // first.  Each 64-deep K half accumulates into its own TMEM columns (the
      // epilogue adds the two in fp32): shorter accumulation chains keep the tensor
      // core's fp32 sums at the accuracy of an FMA chain.
      constexpr int kPairs[6][2] = {{2, 0}, {1, 1}, {0, 2}, {1, 0}, {0, 1}, {0, 0}};
      bool issued = false;
      for (int step = 0; step < F; ++step) {
        if (!mbar_wait(x_ready, step & 1, abort_flag) || !mbar_wait(inv_full, step & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t xa = smem_u32(sX), ib = smem_u32(sI);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
#pragma unroll
          for (int pr = 0; pr < 6; ++pr) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {  // 16 K per MMA: +32 B inside a 128-B row
              const uint32_t koff = kh * 16384 + ks * 32;
              mma_bf16(tmem + kh * 128, desc_k_sw128(xa + kPairs[pr][0] * PLANE + koff),
                       desc_k_sw128(ib + kPairs[pr][1] * PLANE + koff), kIdesc, (pr | ks) != 0);
            }
          }
        }
        issued = true;
        tc_commit(inv_empty);
        tc_commit(acc_full);
      }
      if (*abort_flag && issued) {
        tc_commit(mma_drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(mma_drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // -------------------------------------------------------- state rows
    // Thread = (state row, column quarter): warps 2-17 cover lane quadrant warp % 4
    // (the lanes a warp may read) and column quarter (warp - 2) / 4.  Each thread's
    // whole slice of the B row is requested at the start of the step, before the
    // wait for the previous product: all of its loads are in flight at once.
    constexpr int QC = D / 4;                  // columns per thread
    const int quad = warp & 3;
    const int quarter = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    const int col0 = quarter * QC;
    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + col0;
    float* const banks = dir == 0 ? p.prefix : p.suffix;
    // This warp's 32 rows x 32 columns of the bank of step s's frame.
    auto bank_rows = [&](int s) {
      return reinterpret_cast<uint32_t*>(banks + (((int64_t)frame(s) * H + h) * D + quad * 32) * D + col0);
    };
    uint32_t prev[QC];                         // this quarter row of the state, fp32 bits
    if (p.seed) {
      const uint4* s4 = reinterpret_cast<const uint4*>(p.seed + ((int64_t)h * D + row) * D + col0);
#pragma unroll
      for (int i = 0; i < QC / 4; ++i) {
        const uint4 v = s4[i];
        prev[4 * i] = v.x; prev[4 * i + 1] = v.y; prev[4 * i + 2] = v.z; prev[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < QC; ++i) prev[i] = 0u;
    }
    for (int step = 0; step <= F; ++step) {
      const int fr = frame(step < F ? step : F - 1);
      float4 bq[QC / 4];
      if (!BH && step < F) {
        const float4* b4 = reinterpret_cast<const float4*>(p.B + (((int64_t)fr * H + h) * D + row) * D + col0);
#pragma unroll
        for (int i = 0; i < QC / 4; ++i) bq[i] = b4[i];
      }
      if (step > 0) {
        // P of the previous step: TMEM -> registers -> its bank row.  tcgen05.ld is
        // warp-collective, so a warp proceeds only if none of its lanes gave up.
        if (!__all_sync(0xffffffffu, mbar_wait(acc_full, (step - 1) & 1, abort_flag))) break;
        tc_fence_after();
        uint32_t hi[QC];
        tmem_ld_32x32b_x32(taddr, prev);
        tmem_ld_32x32b_x32(taddr + 128, hi);
        tmem_ld_wait();
        tc_fence_before();
#pragma unroll
        for (int i = 0; i < QC; i += 2) {
          float s0, s1;
          f2_unpack(f2_add(f2_pack(__uint_as_float(prev[i]), __uint_as_float(prev[i + 1])),
                           f2_pack(__uint_as_float(hi[i]), __uint_as_float(hi[i + 1]))), s0, s1);
          prev[i] = __float_as_uint(s0);
          prev[i + 1] = __float_as_uint(s1);
        }
      }
      if (step == F) {
        store_warp_rows_32x32(bank_rows(step - 1), D, prev, lane);
        break;
      }
      if (BH) {  // this thread's 32 values of B_f's row from the staged tile
        if (!__all_sync(0xffffffffu, mbar_wait(b_full, step & 1, abort_flag))) break;
#pragma unroll
        for (int j = 0; j < QC / 8; ++j) {
          const int chunk = col0 / 8 + j;    // 16-byte chunk of the row (8 bf16)
          const uint4 w = *reinterpret_cast<const uint4*>(sB + (chunk >> 3) * (BTILE / 2) + row * 128 +
                                                          (((chunk & 7) ^ (row & 7)) << 4));
          float f8[8];
          unpack8(w, f8);
          bq[2 * j] = make_float4(f8[0], f8[1], f8[2], f8[3]);
          bq[2 * j + 1] = make_float4(f8[4], f8[5], f8[6], f8[7]);
        }
      }
      // X = P diag(alpha_f) + B_f, split into three bf16 parts in the A operand.
      const float* al = BH ? sAl + col0 : alpha_smem ? sAlpha + fr * D + col0 : p.alpha + ((int64_t)fr * H + h) * D + col0;
#pragma unroll
      for (int c = 0; c < QC / 8; ++c) {
        const float4 al0 = *reinterpret_cast<const float4*>(al + 8 * c);
        const float4 al1 = *reinterpret_cast<const float4*>(al + 8 * c + 4);
        const float4 b0 = bq[2 * c], b1 = bq[2 * c + 1];
        const float alv[8] = {al0.x, al0.y, al0.z, al0.w, al1.x, al1.y, al1.z, al1.w};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float x[8];
#pragma unroll
        for (int k = 0; k < 8; k += 2)
          f2_unpack(f2_fma(f2_pack(__uint_as_float(prev[8 * c + k]), __uint_as_float(prev[8 * c + k + 1])),
                           f2_pack(alv[k], alv[k + 1]), f2_pack(bv[k], bv[k + 1])),
                    x[k], x[k + 1]);
        uint32_t w[3][4];
        split3_bf16x8(x, w);
        const uint32_t off = oper_off(row, quarter * (QC / 8) + c);
#pragma unroll
        for (int part = 0; part < 3; ++part)
          *reinterpret_cast<uint4*>(sX + part * PLANE + off) = make_uint4(w[part][0], w[part][1], w[part][2], w[part][3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(x_ready);
        if (BH) mbar_arrive(b_empty);  // done with B_f and alpha_f
      }
      // P_{f-1} to its bank while the tensor cores compute P_f.
      if (step > 0) store_warp_rows_32x32(bank_rows(step - 1), D, prev, lane);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 256);
  }
  if (tid == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}


}  // namespace vscan

// B: fp32 [F, H, d, d]; or, with b_bf16, the same values in bf16 [F, H, d, d].
int launch_scan_tc(const void* inv_planes, const float* B, int b_bf16, const float* alpha, const float* seed,
                   int F, int H, float* prefix, float* suffix, int* status, cudaStream_t stream) {
  using namespace vscan;
  VDN_CHECK_ARG(F >= 1 && H >= 1, "positive F and H required");
  VDN_CHECK_ARG(inv_planes && B && alpha && prefix && suffix, "null pointer");
  VDN_CHECK_ARG(aligned16(inv_planes) && aligned16(B) && aligned16(alpha) && (!seed || aligned16(seed)),
                "scan operands must be 16-byte aligned");
  VDN_CHECK_ARG(aligned32(prefix) && aligned32(suffix), "scan banks must be 32-byte aligned");
  static bool attr_set[2] = {false, false};
  Params p{static_cast<const uint8_t*>(inv_planes), B, alpha, seed, prefix, suffix, F, H, status};
  CUtensorMap tb;
  if (b_bf16) {
    cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)F * H * D};
    cuuint64_t strides[1] = {(cuuint64_t)D * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)D};
    if (int rc = encode_map(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, B, dims, strides, box)) return rc;
    if (!attr_set[1]) {
      VDN_CUDA_TRY(cudaFuncSetAttribute(scan_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)SMEM_BH));
      attr_set[1] = true;
    }
    scan_tc_kernel<true><<<2 * H, THREADS, SMEM_BH, stream>>>(tb, p);
    VDN_LAUNCH_CHECK("vda scan (tcgen05, bf16 B)");
    return VDN_OK;
  }
  std::memset(&tb, 0, sizeof(tb));
  if (!attr_set[0]) {
    VDN_CUDA_TRY(cudaFuncSetAttribute(scan_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
    attr_set[0] = true;
  }
  scan_tc_kernel<false><<<2 * H, THREADS, SMEM, stream>>>(tb, p);
  VDN_LAUNCH_CHECK("vda scan (tcgen05)");
  return VDN_OK;
}

}  // namespace vdn
