// bf16 tcgen05 GEMM with the gate epilogue of the hybrid block:
//     y[:rows, :n] = act(bf16(x @ w^T + bias)),  act = sigmoid (then bf16) on columns < n_sig
// i.e. an eager bf16 nn.Linear (fp32 accumulation, bias added before the one rounding)
// followed by torch.sigmoid on the bf16 result, for the first n_sig output columns.
// The block calls it twice per forward (reference hybrid_attention.py:108-255 and
// attention_gates.py:13-55, branch.py beta_proj):
//   * y1 [T, 5120] @ [softmax_gate; beta_proj; output_gate.down]^T -> [T, 2H + r],
//     sigmoid on the 2H gate columns, the output gate's hidden r columns plain;
//   * hidden [T, r] @ output_gate.up^T + up.bias -> sigmoid -> the VDA gate [T, H*d].
//
// Persistent and warp-specialised, one CTA per SM walking 128 x 256 output tiles
// (N fastest, so a row tile's x stays in L2 while the N tiles sweep):
//   warp 0 lane 0   TMA producer: x tile 128 x 64 and w tile 256 x 64 (bf16, 128B
//                   swizzle; w rows past n read as zero) into a 4-stage ring
//   warp 1          TMEM (512 columns: two 256-column accumulators); lane 0 issues
//                   four 128x256x16 MMAs per stage
//   warps 2-17      epilogue: warp = TMEM lane quadrant x 64-column group; its 32
//                   rows x 64 columns (tcgen05.ld, bias, bf16, sigmoid, bf16) are
//                   written into a 4 KB shared buffer (128-byte swizzle) and sent by
//                   one TMA store; the buffer is reused one tile later, so the store
//                   never holds up the next tile's math (columns past n and rows past
//                   `rows` are clipped by the tensor map).  Sixteen warps, four per
//                   sub-partition, and the bias loaded before the accumulator wait:
//                   the sigmoid's two MUFU operations per element are the kernel's
//                   limit at K = 128, and with fewer warps their latency was.
// Every wait is bounded; a timeout aborts all roles and reports VDN_ERR_TIMEOUT.
// No TMA multicast.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace vdn {
namespace ggemm {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64;   // BK: 64 bf16 = one 128-byte swizzle row
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;           // 16 KB
constexpr int B_BYTES = BN * BK * 2;           // 32 KB
constexpr int THREADS = 576;                   // 2 + 16 epilogue warps
constexpr int PIECE_BYTES = 32 * 128;          // 32 rows x 64 bf16 (one 128B-swizzled store box)
constexpr int EPI_WARPS = 16;
constexpr int NBAR = 2 * STAGES + 2 * 2 + 1;
constexpr size_t SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + EPI_WARPS * PIECE_BYTES + EPI_WARPS * 256 + NBAR * 8 + 64;
static_assert(SMEM <= 232448, "shared memory per CTA");

struct Params {
  const uint16_t* bias;  // [n] bf16 or null
  int64_t rows, n;
  int n_sig;
  int m_tiles, n_tiles, k_blocks;
  int* status;
};

// The sigmoid of a full 8-column chunk runs in pairs (sigmoid_pair: three MUFU operations
// and a few f32x2 instructions per pair, within a few fp32 ulps before the bf16 rounding:
// the up projection 0.162 -> 0.109 ms at config 3 against sigmoid_nr for every element);
// a chunk the gated range ends inside uses sigmoid_nr (common.cuh) per element.
__device__ __forceinline__ float sigmoid_f(float x) { return sigmoid_nr(x); }

// sigmoid of two values: t = 2^(-|x| log2 e) in (0, 1], sigma = 1/(1+t) for x >= 0 and
// t/(1+t) below; both reciprocals from one MUFU reciprocal of (1+t0)(1+t1) in (1, 4].
__device__ __forceinline__ void sigmoid_pair(float& x0, float& x1) {
  const float n0 = __uint_as_float(__float_as_uint(x0) | 0x80000000u);
  const float n1 = __uint_as_float(__float_as_uint(x1) | 0x80000000u);
  float t0, t1;
  f2_unpack(f2_mul(f2_pack(n0, n1), f2_pack(1.4426950408889634f, 1.4426950408889634f)), t0, t1);
  t0 = ex2_approx(t0);
  t1 = ex2_approx(t1);
  float a, b;
  f2_unpack(f2_add(f2_pack(t0, t1), f2_pack(1.0f, 1.0f)), a, b);
  const float r = rcp_approx(a * b);
  float s0, s1;
  f2_unpack(f2_mul(f2_pack(b, a), f2_pack(r, r)), s0, s1);
  x0 = x0 >= 0.f ? s0 : t0 * s0;
  x1 = x1 >= 0.f ? s1 : t1 * s1;
}

__global__ void __launch_bounds__(THREADS, 1)
    gate_gemm_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw,
                     const __grid_constant__ CUtensorMap ty, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* pieces = sB + STAGES * B_BYTES;       // 16 x 4 KB, 1024-aligned
  float* bias_s = reinterpret_cast<float*>(pieces + EPI_WARPS * PIECE_BYTES);   // 64 floats per epilogue warp
  uint64_t* full = reinterpret_cast<uint64_t*>(pieces + EPI_WARPS * PIECE_BYTES + EPI_WARPS * 256);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS);  // one arrival per epilogue warp
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tx);
    prefetch_tensormap(&tw);
    prefetch_tensormap(&ty);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0, pend = 0, pend_phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        const int mb = t / p.n_tiles, nb = t % p.n_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tx, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * B_BYTES, &tw, &full[stage], kb * BK, nb * BN);
          pend |= 1u << stage;
          pend_phase = (pend_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {  // copies already issued land before the CTA may exit
        for (int s = 0; s < STAGES; ++s) {
          if (!(pend >> s & 1)) continue;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full[s], (pend_phase >> s) & 1) && globaltimer() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ----------------------------------------------------------------- MMA
      constexpr uint32_t kIdesc = idesc_bf16(BM, BN, 0, 0);
      int stage = 0, k = 0;
      uint32_t phase = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++k) {
        const int b = k & 1;
        if (!mbar_wait(&acc_empty[b], ((k >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES), b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks)
            mma_bf16(tmem + b * BN, desc_k_sw128(a0 + ks * 32), desc_k_sw128(b0 + ks * 32), kIdesc,
                     (kb | ks) != 0);
          issued = true;
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[b]);
      }
      if (*abort_flag && issued) {
        tc_commit(mma_drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(mma_drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3, group = (warp - 2) >> 2;   // TMEM lane quadrant, 64-column group
    uint8_t* buf = pieces + (warp - 2) * PIECE_BYTES;
    uint8_t* row_base = buf + lane * 128;
    int k = 0;
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++k) {
      const int mb = t / p.n_tiles, nb = t % p.n_tiles, b = k & 1;
      const int64_t row0 = (int64_t)mb * BM + quad * 32;
      const int64_t col0 = (int64_t)nb * BN + group * 64;
      // lane j loads the bias of columns col0 + j and col0 + 32 + j while the tile's MMAs
      // run and parks it in the warp's 64-float slot; every lane then reads eight at a
      // time (broadcast shared loads instead of a shuffle per element)
      const float bj0 = (p.bias && col0 + lane < p.n) ? bf16_bits_to_f32(p.bias[col0 + lane]) : 0.f;
      const float bj1 = (p.bias && col0 + 32 + lane < p.n) ? bf16_bits_to_f32(p.bias[col0 + 32 + lane]) : 0.f;
      float* sb = bias_s + (warp - 2) * 64;
      __syncwarp();
      sb[lane] = bj0;
      sb[32 + lane] = bj1;
      __syncwarp();
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[b], (k >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + b * BN + group * 64;
      const bool live = row0 < p.rows && col0 < p.n;   // warp-uniform
      if (live) {
        if (lane == 0) bulk_wait_group_read<0>();  // the previous tile's store has left the buffer
        __syncwarp();
      }
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {            // 32 columns at a time
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + sub * 32, r);
        tmem_ld_wait();
        if (!live) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 ba = *reinterpret_cast<const float4*>(sb + sub * 32 + c * 8);
          const float4 bb = *reinterpret_cast<const float4*>(sb + sub * 32 + c * 8 + 4);
          const float bv[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[c * 8 + i]) + bv[i];
#pragma unroll
          for (int i = 0; i < 8; i += 2) round_bf16_pair(v[i], v[i + 1]);   // the Linear's bf16 output
          const int64_t c8 = col0 + sub * 32 + c * 8;
          if (c8 + 8 <= p.n_sig) {                   // all eight columns gated
#pragma unroll
            for (int i = 0; i < 8; i += 2) sigmoid_pair(v[i], v[i + 1]);
          } else if (c8 < p.n_sig) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (c8 + i < p.n_sig) v[i] = sigmoid_f(v[i]);
          }
          const uint32_t chunk = sub * 4 + c;        // 16-byte chunk within the 128-byte row
          *reinterpret_cast<uint4*>(row_base + ((chunk ^ (lane & 7)) << 4)) = pack8(v);   // rounds to bf16
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (live) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&ty, buf, (int)col0, (int)row0);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();  // every store written before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}

}  // namespace ggemm
}  // namespace vdn

using namespace vdn;

extern "C" int vdn_gate_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                             int64_t rows, int64_t n, int64_t k, int64_t n_sig, void* y, int64_t ldy,
                             int* status, cudaStream_t stream) {
  using namespace vdn::ggemm;
  VDN_CHECK_ARG(rows >= 0 && n > 0 && k > 0 && k % BK == 0, "need rows >= 0, n > 0 and k a positive multiple of 64");
  VDN_CHECK_ARG(n_sig >= 0 && n_sig <= n, "n_sig must lie in [0, n]");
  VDN_CHECK_ARG(rows < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), "extents too large");
  if (rows == 0) return VDN_OK;
  VDN_CHECK_ARG(x && w && y, "null pointer");
  VDN_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(y), "x, w and y must be 16-byte aligned");
  VDN_CHECK_ARG(ldx >= k && ldw >= k && ldy >= n && ldx % 8 == 0 && ldw % 8 == 0 && ldy % 8 == 0,
                "row strides must cover the extents and be multiples of 8 elements");
  CUtensorMap mx, mw, my;
  {
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    cuuint32_t box[2] = {BK, BM};
    if (int rc = encode_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box)) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)ldw * 2};
    cuuint32_t box[2] = {BK, BN};
    if (int rc = encode_map(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box)) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ldy * 2};
    cuuint32_t box[2] = {64, 32};
    if (int rc = encode_map(&my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box)) return rc;
  }
  Params p;
  p.bias = static_cast<const uint16_t*>(bias);
  p.rows = rows;
  p.n = n;
  p.n_sig = (int)n_sig;
  p.m_tiles = (int)((rows + BM - 1) / BM);
  p.n_tiles = (int)((n + BN - 1) / BN);
  p.k_blocks = (int)(k / BK);
  p.status = status;
  static bool attr_set[64] = {};
  int dev = 0, sms = 148;
  VDN_CUDA_TRY(cudaGetDevice(&dev));
  VDN_CHECK_ARG(dev >= 0 && dev < 64, "device index out of range");
  if (!attr_set[dev]) {
    VDN_CUDA_TRY(cudaFuncSetAttribute(gate_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM));
    attr_set[dev] = true;
  }
  VDN_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  const int grid = tiles < sms ? (int)tiles : sms;
  gate_gemm_kernel<<<grid, THREADS, SMEM, stream>>>(mx, mw, my, p);
  VDN_LAUNCH_CHECK("gate gemm");
  return VDN_OK;
}
