// Block-scaled MXFP8 GEMM on sm_100a tensor cores (tcgen05 kind::mxf8f6f4,
// one E8M0 scale per 32 K-elements):
//     y[:rows_out, :n] = bf16( dequant(xq, xs) @ dequant(wq, ws)^T ) (+ bias)
//
// Persistent, warp-specialised CTA (320 threads, one per SM):
//   warp 0     TMA producer: A tile 128x128 B and B tile 256x128 B (128B swizzle)
//              plus the tile's scale atoms (512-byte bulk copies: the swizzled
//              SWIZZLE_32_4_4 scale layout stores one 128-row x 128-K atom
//              contiguously) into a 4-stage shared-memory ring
//   warp 1     TMEM allocator and single-thread MMA issuer: per stage, three
//              tcgen05.cp (scales -> TMEM) and four 128x256x32 block-scaled MMAs
//              into a 128-lane x 256-column fp32 TMEM accumulator
//   warps 2-9  epilogue: tcgen05.ld of the accumulator (each warp a 32-lane
//              quadrant x 128 columns) into registers, immediate release of
//              the accumulator, then bf16 rounding, bias, gated residual and
//              16-byte stores overlapped with the next tile's MMAs
// Tiles are walked in groups of 16 M-tiles with N fastest so the live A and B
// tiles of all CTAs stay in L2.  Every mbarrier wait is bounded (2 s); a
// timeout aborts all roles, drains copies in flight, frees TMEM and reports
// VDN_ERR_TIMEOUT through `status`.  No TMA multicast is used.
#include "common.cuh"
#include "mxfp8.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <mutex>
#include <stdlib.h>

namespace vdn {
namespace gemm {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;              // 16 KB
constexpr int B_BYTES = BN * BK;              // 32 KB
constexpr int SF_STAGE = 512 * 3;             // SFA atom + two SFB atoms
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0;
constexpr int SF_COL = 256;                   // 12 columns per stage: SFA 4, SFB 8
constexpr int GROUP_M = 16;
constexpr int THREADS = 320;
constexpr int STAGE_PITCH = 80;                // staged epilogue row: 64 B + 16 B pad
constexpr int STAGE_BYTES = 32 * STAGE_PITCH;  // per epilogue warp
constexpr size_t BAR_BYTES = 256;              // mbarriers, TMEM address, abort flag
constexpr size_t SMEM_BYTES =
    1024 + STAGES * (A_BYTES + B_BYTES + SF_STAGE) + BAR_BYTES + 8 * STAGE_BYTES;
static_assert((2 * STAGES + 3) * 8 + 8 <= BAR_BYTES, "barrier region");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");

struct Params {
  const uint8_t* xs;
  const uint8_t* ws;
  const uint8_t* xs2;        // second K range (k_blocks2 > 0): scales of A2 / B2
  const uint8_t* ws2;
  const uint16_t* bias;
  const uint16_t* resid;     // optional epilogue: y = resid + gate[col] * result
  const uint16_t* gate;
  int64_t ldr;
  uint16_t* y;
  int64_t ldy;
  int64_t rows_out;
  int64_t n;
  int m_tiles, n_tiles, k_blocks, k_blocks2, n_groups;  // n_groups = n_pad / 128
  int vec_ok;                // 16-byte vector epilogue allowed (alignment of y / bias / resid / gate)
  int tma_y;                 // pair kernel, plain / residual store: y leaves by TMA stores (tmap_y)
  // Scatter epilogue (chunk_dst != null): the 128 output columns of chunk c go to
  // chunk_dst[c] + (dst_row0 + row) * dst_ld, e.g. each head's q / k / v slice
  // straight into the receive buffer of the rank that owns the head.
  const uint64_t* chunk_dst;
  int64_t dst_ld;
  int64_t dst_row0;
  // Activation-quantise epilogue (q_out != null): y = act(bf16(acc + bias)) rounded
  // to bf16, then MXFP8 codes q_out [m_pad, n] and swizzled scales s_out; rows
  // in [rows_out, m_pad) get zero codes and scales.
  int act;
  uint8_t* q_out;
  uint8_t* s_out;
  int* status;
};

__device__ __forceinline__ void tile_coords_g(int t, int m_tiles, int n_tiles, int group, int& mb,
                                              int& nb) {
  const int per_group = group * n_tiles;
  const int g = t / per_group;
  const int first = g * group;
  const int gsize = min(group, m_tiles - first);
  const int local = t - g * per_group;
  mb = first + local % gsize;
  nb = local / gsize;
}

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mb, int& nb) {
  const int per_group = GROUP_M * n_tiles;
  const int g = t / per_group;
  const int first = g * GROUP_M;
  const int gsize = min(GROUP_M, m_tiles - first);
  const int local = t - g * per_group;
  mb = first + local % gsize;
  nb = local / gsize;
}

__device__ __forceinline__ void prefetch_l2_row(const uint16_t* ptr, int64_t cols) {
  const char* c = reinterpret_cast<const char*>(ptr);
  for (int64_t off = 0; off < cols * 2; off += 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(c + off));
}

// One thread's row segment of the epilogue: y = bf16(acc) (+ bias, rounded to
// bf16) and, with a residual, y = resid + bf16(gate * y), rounded to bf16.
// Bias, gate and residual are read through the read-only path: y must not
// overlap them.
__device__ __forceinline__ void store_row(const Params& p, const uint32_t (&r)[128], int64_t row,
                                          int64_t col0) {
  uint16_t* dst = p.y + row * p.ldy + col0;
  if (p.vec_ok && col0 + 128 <= p.n) {
    const uint4* rrow = p.resid ? reinterpret_cast<const uint4*>(p.resid + row * p.ldr + col0) : nullptr;
    const uint4* bias = p.bias ? reinterpret_cast<const uint4*>(p.bias + col0) : nullptr;
    const uint4* gate = p.resid ? reinterpret_cast<const uint4*>(p.gate + col0) : nullptr;
    uint4* dst4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        v[i] = __uint_as_float(r[8 * j + i]);
        v[i + 1] = __uint_as_float(r[8 * j + i + 1]);
        round_bf16_pair(v[i], v[i + 1]);
      }
      if (bias) {
        float b[8];
        unpack8(__ldg(bias + j), b);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          v[i] += b[i];
          v[i + 1] += b[i + 1];
          round_bf16_pair(v[i], v[i + 1]);
        }
      }
      if (rrow) {
        float g[8], x[8];
        unpack8(__ldg(gate + j), g);
        unpack8(__ldg(rrow + j), x);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float a = g[i] * v[i], b = g[i + 1] * v[i + 1];
          round_bf16_pair(a, b);
          v[i] = x[i] + a;
          v[i + 1] = x[i + 1] + b;
        }
      }
      dst4[j] = pack8(v);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 128; ++i) {
    const int64_t col = col0 + i;
    if (col < p.n) {
      float v = round_bf16(__uint_as_float(r[i]));
      if (p.bias) v = round_bf16(v + bf16_bits_to_f32(p.bias[col]));
      if (p.resid)
        v = bf16_bits_to_f32(p.resid[row * p.ldr + col]) + round_bf16(bf16_bits_to_f32(p.gate[col]) * v);
      dst[i] = f32_to_bf16_bits(v);
    }
  }
}

// Bulk-store form of store_row for one warp (32 consecutive rows from row0, 128
// columns from col0, n % 128 == 0): the same arithmetic, but each 32-column piece of
// the warp's rows is written into a 32 x 64-byte bf16 buffer in shared memory
// (64-byte swizzle: the 32 row writers hit distinct banks) and leaves by one TMA
// store, instead of 16-byte stores that touch 32 rows per instruction.  Rows past
// rows_out are clipped by the tensor map.  The buffer is refilled once the previous
// piece's store has read it (buf 512-byte aligned: the swizzle phase is the row's).
__device__ __forceinline__ void store_rows_tma(const Params& p, const CUtensorMap* ymap, const uint32_t (&r)[128],
                                               int64_t row0, int lane, int64_t col0, uint8_t* buf) {
  const int64_t row = row0 + lane;
  const uint4* rrow = (p.resid && row < p.rows_out) ? reinterpret_cast<const uint4*>(p.resid + row * p.ldr + col0)
                                                    : nullptr;
  const uint4* bias = p.bias ? reinterpret_cast<const uint4*>(p.bias + col0) : nullptr;
  const uint4* gate = p.resid ? reinterpret_cast<const uint4*>(p.gate + col0) : nullptr;
  uint8_t* mine = buf + lane * 64;
  const uint32_t phase = (lane >> 1) & 3;
#pragma unroll
  for (int piece = 0; piece < 4; ++piece) {
    uint4 out[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = 4 * piece + jj;
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        v[i] = __uint_as_float(r[8 * j + i]);
        v[i + 1] = __uint_as_float(r[8 * j + i + 1]);
        round_bf16_pair(v[i], v[i + 1]);
      }
      if (bias) {
        float b[8];
        unpack8(__ldg(bias + j), b);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          v[i] += b[i];
          v[i + 1] += b[i + 1];
          round_bf16_pair(v[i], v[i + 1]);
        }
      }
      if (gate) {
        float g[8], x[8];
        unpack8(__ldg(gate + j), g);
        if (rrow) {
          unpack8(__ldg(rrow + j), x);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = 0.f;  // a clipped row
        }
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float a = g[i] * v[i], b = g[i + 1] * v[i + 1];
          round_bf16_pair(a, b);
          v[i] = x[i] + a;
          v[i + 1] = x[i + 1] + b;
        }
      }
      out[jj] = pack8(v);
    }
    if (lane == 0) bulk_wait_group_read<0>();  // the previous piece has left the buffer
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(mine + ((c ^ phase) << 4)) = out[c];
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(ymap, buf, (int)(col0 + 32 * piece), (int)row0);
      bulk_commit_group();
    }
  }
}

// Activation-quantise epilogue of one thread's row segment (128 columns = four
// MXFP8 blocks): the same arithmetic as the unfused bf16 store followed by the
// activation quantiser, so codes and scales are bit-identical to that path.
template <bool GELU>
__device__ __forceinline__ void store_row_quant(const Params& p, const uint32_t (&r)[128], int64_t row,
                                                int64_t col0) {
  const bool valid = row < p.rows_out;
  const uint4* bias = p.bias ? reinterpret_cast<const uint4*>(p.bias + col0) : nullptr;
  uint32_t word = 0;
#pragma unroll
  for (int blk = 0; blk < 4; ++blk) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float* w = v + 8 * j;
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        w[i] = __uint_as_float(r[32 * blk + 8 * j + i]);
        w[i + 1] = __uint_as_float(r[32 * blk + 8 * j + i + 1]);
        round_bf16_pair(w[i], w[i + 1]);
      }
      if (bias) {
        float b[8];
        unpack8(__ldg(bias + 4 * blk + j), b);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          w[i] += b[i];
          w[i + 1] += b[i + 1];
          round_bf16_pair(w[i], w[i + 1]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float a = v[i];
      if (GELU) a = round_bf16(gelu_tanh(a));
      v[i] = valid ? a : 0.f;
    }
    uint32_t amax_bits = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint32_t b = __float_as_uint(v[i]) & 0x7FFFFFFFu;
      amax_bits = b > amax_bits ? b : amax_bits;
    }
    float inv;
    const uint32_t sbyte = e8m0_from_amax_bits(amax_bits, &inv);
    word |= sbyte << (8 * blk);
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      packed[i] = e4m3x4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv, v[4 * i + 3] * inv);
    uint4* qp = reinterpret_cast<uint4*>(p.q_out + row * p.n + col0 + 32 * blk);
    qp[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    qp[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
  *reinterpret_cast<uint32_t*>(p.s_out + scale_offset(row, col0 >> 5, p.n)) = word;
}

// Scatter epilogue of one warp (32 consecutive rows from row0, 128 columns from
// col0): bf16(acc) (+ bias), then the rows leave through a 32 x 32-column
// shared-memory transpose so that every store instruction writes 64-byte row
// pieces (four lanes x 16 B) of the destination instead of 16 bytes of 32
// different rows: peer stores over NVLink want contiguous runs.  Host checks
// guarantee n % 128 == 0 and 16-byte alignment.
__device__ __forceinline__ void store_rows_staged(const Params& p, const uint32_t (&r)[128], int64_t row0,
                                                  int lane, int64_t col0, uint8_t* stage) {
  const uint4* bias = p.bias ? reinterpret_cast<const uint4*>(p.bias + col0) : nullptr;
  uint16_t* base = reinterpret_cast<uint16_t*>(p.chunk_dst[col0 >> 7]);
  uint4* mine = reinterpret_cast<uint4*>(stage + lane * STAGE_PITCH);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      v[i] = __uint_as_float(r[8 * j + i]);
      v[i + 1] = __uint_as_float(r[8 * j + i + 1]);
      round_bf16_pair(v[i], v[i + 1]);
    }
    if (bias) {
      float b[8];
      unpack8(__ldg(bias + j), b);
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        v[i] += b[i];
        v[i + 1] += b[i + 1];
        round_bf16_pair(v[i], v[i + 1]);
      }
    }
    mine[j & 3] = pack8(v);
    if ((j & 3) == 3) {
      __syncwarp();
      const int q = lane & 3;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rl = i * 8 + (lane >> 2);
        const uint4 val = *reinterpret_cast<const uint4*>(stage + rl * STAGE_PITCH + q * 16);
        const int64_t row = row0 + rl;
        if (row < p.rows_out)
          *reinterpret_cast<uint4*>(base + (p.dst_row0 + row) * p.dst_ld + (j >> 2) * 32 + q * 8) = val;
      }
      __syncwarp();
    }
  }
}

// Epilogue kinds, one kernel instantiation each (keeps every variant's code small).
enum Epilogue { EPI_STORE = 0, EPI_SCATTER = 1, EPI_QUANT = 2, EPI_QUANT_GELU = 3 };

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    mxfp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_a2,
                      const __grid_constant__ CUtensorMap tmap_b2, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sSF = sB + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSF + STAGES * SF_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint8_t* stage_base = sSF + STAGES * SF_STAGE + BAR_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
    if (p.k_blocks2) {
      prefetch_tensormap(&tmap_a2);
      prefetch_tensormap(&tmap_b2);
    }
  }
  if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pending = 0;            // stages with loads issued (bit mask)
      uint32_t pending_phase = 0;      // the full-barrier parity those loads complete
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, p.m_tiles, p.n_tiles, mb, nb);
        const bool has_b1 = 2 * nb + 1 < p.n_groups;
        const int kb_total = p.k_blocks + p.k_blocks2;
        for (int kbt = 0; kbt < kb_total; ++kbt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
          // K blocks of the first operand pair, then of the second (K concatenation).
          const bool second = kbt >= p.k_blocks;
          const int kb = second ? kbt - p.k_blocks : kbt;
          const int kbn = second ? p.k_blocks2 : p.k_blocks;
          const CUtensorMap* ma = second ? &tmap_a2 : &tmap_a;
          const CUtensorMap* mbm = second ? &tmap_b2 : &tmap_b;
          const uint8_t* xs = second ? p.xs2 : p.xs;
          const uint8_t* ws = second ? p.ws2 : p.ws;
          const uint32_t bytes = A_BYTES + B_BYTES + (has_b1 ? 3 : 2) * 512;
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(sA + stage * A_BYTES, ma, &full[stage], kb * BK, mb * BM);
          tma_load_2d(sB + stage * B_BYTES, mbm, &full[stage], kb * BK, nb * BN);
          uint8_t* sf = sSF + stage * SF_STAGE;
          bulk_load(sf, xs + ((int64_t)mb * kbn + kb) * 512, 512, &full[stage]);
          bulk_load(sf + 512, ws + ((int64_t)(2 * nb) * kbn + kb) * 512, 512, &full[stage]);
          if (has_b1)
            bulk_load(sf + 1024, ws + ((int64_t)(2 * nb + 1) * kbn + kb) * 512, 512, &full[stage]);
          pending |= 1u << stage;
          pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag) {
        // Let every copy already issued land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s) {
          if (!(pending >> s & 1)) continue;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full[s], (pending_phase >> s) & 1) &&
                 globaltimer() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ----------------------------------------------------------------- MMA
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        if (!mbar_wait(acc_empty, acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        bool ok = true;
        const int kb_total = p.k_blocks + p.k_blocks2;
        for (int kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf_a = tmem + SF_COL + stage * 12;
          const uint32_t sf_b = sf_a + 4;
          const uint32_t sf_smem = smem_u32(sSF + stage * SF_STAGE);
          tmem_cp_32x128_x4(sf_a, desc_sf_atom(sf_smem));
          tmem_cp_32x128_x4(sf_b, desc_sf_atom(sf_smem + 512));
          tmem_cp_32x128_x4(sf_b + 4, desc_sf_atom(sf_smem + 1024));
          const uint64_t adesc = desc_k_sw128(smem_u32(sA + stage * A_BYTES));
          const uint64_t bdesc = desc_k_sw128(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            // +32 bytes along K inside the 128-byte swizzled row: +2 in start>>4.
            mma_mxf8(tmem + ACC_COL, adesc + 2 * k, bdesc + 2 * k, idesc_mxf8(BM, BN, k),
                     sf_a | ((uint32_t)k << 30), sf_b | ((uint32_t)k << 30), (kb | k) != 0);
          }
          issued = true;
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(acc_full);
        acc_phase ^= 1;
      }
      if (*abort_flag && issued) {
        // Wait for every MMA / copy issued so far before TMEM is freed.
        tc_commit(mma_done);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(mma_done, 0) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warps 2-9: TMEM lane quadrant warp % 4 (the only lanes a warp may read),
    // column half (warp - 2) / 4.  Each thread owns one output row x 128 columns:
    // it moves them into registers, hands the accumulator back to the MMA warp
    // at once, and finishes bias / residual / stores while the next tile's
    // MMAs run.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, p.m_tiles, p.n_tiles, mb, nb);
      const int64_t row = (int64_t)mb * BM + row_in_tile;
      const int64_t col0 = (int64_t)nb * BN + half * 128;
      const bool live = row < p.rows_out && col0 < p.n;
      if (live && p.resid) prefetch_l2_row(p.resid + row * p.ldr + col0, p.n - col0 < 128 ? p.n - col0 : 128);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, acc_phase, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[128];
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + ACC_COL + half * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(taddr + c * 32, r + 32 * c);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(acc_empty);
      acc_phase ^= 1;
      if constexpr (EPI == EPI_QUANT || EPI == EPI_QUANT_GELU) {
        if (col0 < p.n) store_row_quant<EPI == EPI_QUANT_GELU>(p, r, row, col0);  // zeros past rows_out
      } else if constexpr (EPI == EPI_SCATTER) {
        if (col0 < p.n)  // warp-uniform
          store_rows_staged(p, r, (int64_t)mb * BM + quad * 32, lane, col0,
                            stage_base + (warp - 2) * STAGE_BYTES);
      } else {
        if (live) store_row(p, r, row, col0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}

// ------------------------------------------------------------ CTA-pair kernel
// The same GEMM with a 256 x 256 tile per CTA pair (a cluster of two CTAs on
// neighbouring SMs, tcgen05 cta_group::2): each CTA stages its 128 rows of A and
// its 128-row half of B per 256-deep K block (64 KB; per FLOP a third fewer bytes
// from L2 than the single-CTA tile), the even CTA issues one 256 x 256 x 32
// block-scaled MMA over both CTAs' shared memory per 32 K, and each CTA's TMEM
// receives its own 128 x 256 accumulator.  The 256-deep stage carries six scale
// atoms copied to TMEM back to back ahead of eight MMAs: scale copies and MMAs
// share the tensor pipe in order, and every switch between them costs a bubble.
// Both CTAs' TMA loads (operands and scale atoms, no multicast) signal the
// leader's full barrier; the leader's MMA commits free the stage in both CTAs;
// both CTAs' epilogues drain their own accumulator and report to the leader.
constexpr int P_BK = 256;             // K per stage: two 128-byte swizzled sub-tiles
constexpr int P_STAGES = 3;
constexpr int P_SUB = 128 * 128;      // one 128-row x 128-byte sub-tile
constexpr int P_A_BYTES = 2 * P_SUB;  // 32 KB
constexpr int P_B_BYTES = 2 * P_SUB;  // 32 KB
constexpr int P_SF_STAGE = 512 * 6;   // SFA: 2 K-atoms; SFB: 2 N-halves x 2 K-atoms
constexpr int P_SF_COLS = 24;         // TMEM scale columns per stage
constexpr int P_GROUP_M = 16;        // 256-row tiles per group (4096 rows: measured best of 4 / 8 / 16 / 32)
constexpr size_t P_SMEM_BYTES =
    1024 + P_STAGES * (P_A_BYTES + P_B_BYTES + P_SF_STAGE) + BAR_BYTES + 8 * STAGE_BYTES;
static_assert(P_SMEM_BYTES <= 232448, "shared memory per CTA");
static_assert((2 * P_STAGES + 3) * 8 + 8 <= BAR_BYTES, "barrier region");
static_assert(256 + P_STAGES * P_SF_COLS <= TMEM_COLS, "scale columns");
constexpr uint64_t kDrainNs = 200000;  // abort path: time for a CTA's own copies to land

struct PairMaps {
  CUtensorMap sfa, sfb, sfa2, sfb2;  // scale atoms as [atoms, 128] uint32 rows
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    mxfp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_a2,
                           const __grid_constant__ CUtensorMap tmap_b2,
                           const __grid_constant__ PairMaps sf, const __grid_constant__ CUtensorMap tmap_y,
                           const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + P_STAGES * P_A_BYTES;
  uint8_t* stage_base = sB + P_STAGES * P_B_BYTES;  // 1024-aligned; 8 epilogue buffers of 2560 B
  uint8_t* sSF = stage_base + 8 * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSF + P_STAGES * P_SF_STAGE);
  uint64_t* empty = full + P_STAGES;
  uint64_t* acc_full = empty + P_STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 16);  // one arrival per epilogue warp of both CTAs
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
    prefetch_tensormap(&sf.sfa);
    prefetch_tensormap(&sf.sfb);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barrier inits visible to the peer before any remote arrive / copy
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int num_tiles = p.m_tiles * p.n_tiles;  // m_tiles counts 256-row tiles here

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      const uint32_t full_leader = mapa_shared(full, 0);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pending = 0, pending_phase = 0;
      bool issued = false;
      for (int t = pair_id; t < num_tiles && !*abort_flag; t += npairs) {
        int mb, nb;
        tile_coords_g(t, p.m_tiles, p.n_tiles, P_GROUP_M, mb, nb);
        const bool has_b1 = 2 * nb + 1 < p.n_groups;
        const int kb_total = p.k_blocks + p.k_blocks2;
        for (int kbt = 0; kbt < kb_total; ++kbt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
          const bool second = kbt >= p.k_blocks;
          const int kb = second ? kbt - p.k_blocks : kbt;
          const int kbn = 2 * (second ? p.k_blocks2 : p.k_blocks);  // 128-deep atoms per row block
          const CUtensorMap* ma = second ? &tmap_a2 : &tmap_a;
          const CUtensorMap* mbm = second ? &tmap_b2 : &tmap_b;
          const CUtensorMap* msa = second ? &sf.sfa2 : &sf.sfa;
          const CUtensorMap* msb = second ? &sf.sfb2 : &sf.sfb;
          // kbn counts 128-deep scale atoms; this stage covers atoms 2 kb, 2 kb + 1.
          const uint32_t bytes = P_A_BYTES + P_B_BYTES + (has_b1 ? 6 : 4) * 512;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * bytes);
          const uint32_t fb = full_leader + stage * 8;
          const int arow = (mb * 2 + (int)rank) * 128, brow = (nb * 2 + (int)rank) * 128;
          uint8_t* a_s = sA + stage * P_A_BYTES;
          uint8_t* b_s = sB + stage * P_B_BYTES;
          tma_load_2d_pair(a_s, ma, fb, kb * P_BK, arow);
          tma_load_2d_pair(a_s + P_SUB, ma, fb, kb * P_BK + 128, arow);
          tma_load_2d_pair(b_s, mbm, fb, kb * P_BK, brow);
          tma_load_2d_pair(b_s + P_SUB, mbm, fb, kb * P_BK + 128, brow);
          uint8_t* sfs = sSF + stage * P_SF_STAGE;
          tma_load_2d_pair(sfs, msa, fb, 0, (mb * 2 + (int)rank) * kbn + 2 * kb);
          tma_load_2d_pair(sfs + 1024, msb, fb, 0, (2 * nb) * kbn + 2 * kb);
          if (has_b1) tma_load_2d_pair(sfs + 2048, msb, fb, 0, (2 * nb + 1) * kbn + 2 * kb);
          issued = true;
          pending |= 1u << stage;
          pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && issued) {
        // Let copies already issued land before the CTA can exit.  The leader
        // watches its full barriers; the peer's copies signal the leader's
        // barriers, so it waits a fixed bounded time instead.
        if (leader) {
          for (int s = 0; s < P_STAGES; ++s) {
            if (!(pending >> s & 1)) continue;
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(&full[s], (pending_phase >> s) & 1) && globaltimer() - t0 < kWaitLimitNs) {
            }
          }
        } else {
          const uint64_t t0 = globaltimer();
          while (globaltimer() - t0 < kDrainNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ----------------------------------------------------------------- MMA
      // Per 256-deep stage: six scale-atom copies to TMEM, then eight MMAs.
      // (Copying the next stage's scales ahead of the current MMAs was measured
      // slower: it makes every MMA batch wait for the following stage's data.)
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool issued = false;
      for (int t = pair_id; t < num_tiles; t += npairs) {
        if (!mbar_wait(acc_empty, acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        bool ok = true;
        const int kb_total = p.k_blocks + p.k_blocks2;
        for (int kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // TMEM scale columns of the stage: SFA atom h at +4h; SFB of K-atom h at
          // +8 + 8h (N rows 0-127) and +12 + 8h (N rows 128-255).
          const uint32_t sf = tmem + SF_COL + stage * P_SF_COLS;
          const uint32_t sf_smem = smem_u32(sSF + stage * P_SF_STAGE);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tmem_cp_pair_32x128_x4(sf + 4 * h, desc_sf_atom(sf_smem + 512 * h));
            tmem_cp_pair_32x128_x4(sf + 8 + 8 * h, desc_sf_atom(sf_smem + 1024 + 512 * h));
            tmem_cp_pair_32x128_x4(sf + 12 + 8 * h, desc_sf_atom(sf_smem + 2048 + 512 * h));
          }
          const uint32_t a0 = smem_u32(sA + stage * P_A_BYTES), b0 = smem_u32(sB + stage * P_B_BYTES);
#pragma unroll
          for (int k = 0; k < P_BK / 32; ++k) {
            const int h = k >> 2, kk = k & 3;
            const uint64_t adesc = desc_k_sw128(a0 + h * P_SUB) + 2 * kk;
            const uint64_t bdesc = desc_k_sw128(b0 + h * P_SUB) + 2 * kk;
            mma_mxf8_pair(tmem + ACC_COL, adesc, bdesc, idesc_mxf8(256, BN, kk),
                          (sf + 4 * h) | ((uint32_t)kk << 30), (sf + 8 + 8 * h) | ((uint32_t)kk << 30),
                          (kb | k) != 0);
          }
          issued = true;
          tc_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(acc_full, 0x3);
        acc_phase ^= 1;
      }
      if (*abort_flag && issued) {
        tc_commit_pair(mma_done, 0x1);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(mma_done, 0) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t acc_empty_leader = mapa_shared(acc_empty, 0);
    uint32_t acc_phase = 0;
    for (int t = pair_id; t < num_tiles; t += npairs) {
      int mb, nb;
      tile_coords_g(t, p.m_tiles, p.n_tiles, P_GROUP_M, mb, nb);
      const int64_t row_base = (int64_t)(mb * 2 + (int)rank) * 128;
      const int64_t row = row_base + row_in_tile;
      const int64_t col0 = (int64_t)nb * BN + half * 128;
      const bool live = row < p.rows_out && col0 < p.n;
      if (EPI == EPI_STORE && live && p.resid)
        prefetch_l2_row(p.resid + row * p.ldr + col0, p.n - col0 < 128 ? p.n - col0 : 128);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, acc_phase, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[128];
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + ACC_COL + half * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(taddr + c * 32, r + 32 * c);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(acc_empty);
        else mbar_arrive_cluster(acc_empty_leader);
      }
      acc_phase ^= 1;
      if constexpr (EPI == EPI_QUANT || EPI == EPI_QUANT_GELU) {
        if (col0 < p.n) store_row_quant<EPI == EPI_QUANT_GELU>(p, r, row, col0);
      } else if constexpr (EPI == EPI_SCATTER) {
        if (col0 < p.n) store_rows_staged(p, r, row_base + quad * 32, lane, col0, stage_base + (warp - 2) * STAGE_BYTES);
      } else {
        if (p.tma_y) {
          if (row_base + quad * 32 < p.rows_out && col0 < p.n)
            store_rows_tma(p, &tmap_y, r, row_base + quad * 32, lane, col0, stage_base + (warp - 2) * STAGE_BYTES);
        } else if (live) {
          store_row(p, r, row, col0);
        }
      }
    }
    if (EPI == EPI_STORE && lane == 0) bulk_wait_group<0>();  // stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs and every remote arrive are done in both CTAs
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
  cluster_sync();  // neither CTA leaves while the pair's TMEM or barriers are in use
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}

// -------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

static int make_map(CUtensorMap* map, const void* base, int64_t k_pad, int64_t rows, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)k_pad, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k_pad};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VDN_OK;
}

// bf16 output y [rows_out, n] (row stride ldy) for the bulk-store epilogue: 32 x 32
// boxes with 64-byte swizzle.
static int make_y_map(CUtensorMap* map, const void* y, int64_t n, int64_t rows_out, int64_t ldy) {
  auto fn = encode_fn();
  if (!fn) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows_out};
  cuuint64_t strides[1] = {(cuuint64_t)ldy * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(y), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled (y) failed (%d)", (int)r);
  return VDN_OK;
}

// Scale atoms of a padded operand as a 2D tensor: [atoms, 128] uint32 rows of
// 512 bytes (one SWIZZLE_32_4_4 atom per row), loaded two atoms per copy.
static int make_sf_map(CUtensorMap* map, const void* base, int64_t atoms) {
  auto fn = encode_fn();
  if (!fn) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {128, (cuuint64_t)atoms};
  cuuint64_t strides[1] = {512};
  cuuint32_t box[2] = {128, 2};  // two consecutive K atoms: one 256-deep stage
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled (scales) failed (%d)", (int)r);
  return VDN_OK;
}

struct DeviceInfo {
  int sms = 0;
  int pairs = 0;  // co-resident CTA pairs of the pair kernel (0: pair kernel unavailable)
  bool smem_set = false;
};

static int device_info(DeviceInfo** out) {
  static DeviceInfo info[64];
  static std::mutex mu;
  int dev = 0;
  VDN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(VDN_ERR_RUNTIME, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  DeviceInfo& d = info[dev];
  if (!d.smem_set) {
    VDN_CUDA_TRY(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    VDN_CUDA_TRY(cudaFuncSetAttribute(mxfp8_gemm_kernel<EPI_STORE>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    VDN_CUDA_TRY(cudaFuncSetAttribute(mxfp8_gemm_kernel<EPI_SCATTER>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    VDN_CUDA_TRY(cudaFuncSetAttribute(mxfp8_gemm_kernel<EPI_QUANT>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    VDN_CUDA_TRY(cudaFuncSetAttribute(mxfp8_gemm_kernel<EPI_QUANT_GELU>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    const void* pair_kernels[4] = {(const void*)mxfp8_gemm_pair_kernel<EPI_STORE>,
                                   (const void*)mxfp8_gemm_pair_kernel<EPI_SCATTER>,
                                   (const void*)mxfp8_gemm_pair_kernel<EPI_QUANT>,
                                   (const void*)mxfp8_gemm_pair_kernel<EPI_QUANT_GELU>};
    for (const void* k : pair_kernels)
      VDN_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM_BYTES));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (d.sms / 2), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, (const void*)mxfp8_gemm_pair_kernel<EPI_STORE>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    d.pairs = clusters;
    d.smem_set = true;
  }
  *out = &d;
  return VDN_OK;
}

}  // namespace gemm
}  // namespace vdn

using namespace vdn;

static int launch_gemm(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq, const uint8_t* ws,
                       int64_t k_pad, const uint8_t* xq2, const uint8_t* xs2, const uint8_t* wq2,
                       const uint8_t* ws2, int64_t k_pad2, const void* bias, int64_t m_pad,
                       int64_t n, int64_t n_pad, int64_t rows_out, void* y, int64_t ldy,
                       const void* resid, int64_t ldr, const void* gate, int* status,
                       cudaStream_t stream, const uint64_t* chunk_dst = nullptr,
                       int64_t dst_ld = 0, int64_t dst_row0 = 0, int act = 0,
                       uint8_t* q_out = nullptr, uint8_t* s_out = nullptr) {
  using namespace vdn::gemm;
  VDN_CHECK_ARG(m_pad >= 0 && n > 0 && n_pad > 0 && k_pad > 0 && k_pad2 >= 0, "bad GEMM extents");
  VDN_CHECK_ARG(m_pad % 128 == 0 && n_pad % 128 == 0 && k_pad % 128 == 0 && k_pad2 % 128 == 0,
                "m_pad, n_pad and k_pad must be multiples of 128");
  VDN_CHECK_ARG(n <= n_pad && rows_out >= 0 && rows_out <= m_pad, "crop exceeds the padded extents");
  VDN_CHECK_ARG(chunk_dst || q_out || ldy >= n, "ldy must be at least n");
  VDN_CHECK_ARG(!q_out || (s_out && n % 128 == 0 && !resid && !chunk_dst && aligned16(q_out) &&
                           (reinterpret_cast<uintptr_t>(s_out) & 3) == 0),
                "activation-quantise epilogue needs n % 128 == 0, aligned q / s and no residual");
  VDN_CHECK_ARG(!chunk_dst || (n % 128 == 0 && dst_ld % 8 == 0 && dst_ld >= 128 && dst_row0 >= 0 && !resid),
                "scatter epilogue needs n % 128 == 0, dst_ld % 8 == 0 and no residual");
  VDN_CHECK_ARG(!resid || (gate && ldr >= n), "a residual needs a gate vector and ldr >= n");
  if (rows_out == 0 || m_pad == 0) return VDN_OK;
  VDN_CHECK_ARG(xq && xs && wq && ws && (y || chunk_dst || q_out), "null pointer");
  VDN_CHECK_ARG(aligned16(xq) && aligned16(xs) && aligned16(wq) && aligned16(ws),
                "codes and scales must be 16-byte aligned");
  VDN_CHECK_ARG(k_pad2 == 0 || (xq2 && xs2 && wq2 && ws2 && aligned16(xq2) && aligned16(xs2) &&
                                aligned16(wq2) && aligned16(ws2)),
                "second operand pair must be non-null and 16-byte aligned");
  VDN_CHECK_ARG(m_pad / 128 < (1 << 30) && n_pad / 128 < (1 << 30), "extents too large");
  if (resid) {
    // The epilogue reads the residual through the read-only cache path.
    const uintptr_t y0 = reinterpret_cast<uintptr_t>(y), y1 = y0 + 2 * ((rows_out - 1) * ldy + n);
    const uintptr_t r0 = reinterpret_cast<uintptr_t>(resid), r1 = r0 + 2 * ((rows_out - 1) * ldr + n);
    VDN_CHECK_ARG(y1 <= r0 || r1 <= y0, "y must not overlap the residual");
  }
  DeviceInfo* info = nullptr;
  if (int rc = device_info(&info)) return rc;
  CUtensorMap ma, mb, ma2, mb2;
  if (int rc = make_map(&ma, xq, k_pad, m_pad, BM)) return rc;
  if (int rc = make_map(&mb, wq, k_pad, n_pad, BN)) return rc;
  if (k_pad2) {
    if (int rc = make_map(&ma2, xq2, k_pad2, m_pad, BM)) return rc;
    if (int rc = make_map(&mb2, wq2, k_pad2, n_pad, BN)) return rc;
  } else {
    ma2 = ma;
    mb2 = mb;
  }
  Params p;
  p.xs = xs;
  p.ws = ws;
  p.xs2 = xs2;
  p.ws2 = ws2;
  p.bias = static_cast<const uint16_t*>(bias);
  p.resid = static_cast<const uint16_t*>(resid);
  p.gate = static_cast<const uint16_t*>(gate);
  p.ldr = ldr;
  p.y = static_cast<uint16_t*>(y);
  p.ldy = ldy;
  p.rows_out = rows_out;
  p.n = n;
  p.m_tiles = (int)(m_pad / BM);
  p.n_tiles = (int)((n_pad + BN - 1) / BN);
  p.k_blocks = (int)(k_pad / BK);
  p.k_blocks2 = (int)(k_pad2 / BK);
  p.n_groups = (int)(n_pad / 128);
  p.status = status;
  p.vec_ok = (chunk_dst || q_out ? true : aligned16(y) && ldy % 8 == 0) && (!bias || aligned16(bias)) &&
             (!resid || (aligned16(resid) && ldr % 8 == 0 && aligned16(gate)));
  p.chunk_dst = chunk_dst;
  p.dst_ld = dst_ld;
  p.dst_row0 = dst_row0;
  p.act = act;
  p.q_out = q_out;
  p.s_out = s_out;
  p.tma_y = 0;
  static const bool pair_off = [] {
    const char* e = getenv("VDN_GEMM_PAIR");
    return e && e[0] == '0';
  }();
  if (!pair_off && info->pairs > 0 && m_pad % 256 == 0 && k_pad % 256 == 0 && k_pad2 % 256 == 0) {
    PairMaps sf;
    const int64_t kb1 = k_pad / BK, kb2 = k_pad2 / BK;
    if (int rc = make_map(&ma, xq, k_pad, m_pad, 128)) return rc;
    if (int rc = make_map(&mb, wq, k_pad, n_pad, 128)) return rc;
    if (int rc = make_sf_map(&sf.sfa, xs, (m_pad / 128) * kb1)) return rc;
    if (int rc = make_sf_map(&sf.sfb, ws, (n_pad / 128) * kb1)) return rc;
    if (k_pad2) {
      if (int rc = make_map(&ma2, xq2, k_pad2, m_pad, 128)) return rc;
      if (int rc = make_map(&mb2, wq2, k_pad2, n_pad, 128)) return rc;
      if (int rc = make_sf_map(&sf.sfa2, xs2, (m_pad / 128) * kb2)) return rc;
      if (int rc = make_sf_map(&sf.sfb2, ws2, (n_pad / 128) * kb2)) return rc;
    } else {
      ma2 = ma;
      mb2 = mb;
      sf.sfa2 = sf.sfa;
      sf.sfb2 = sf.sfb;
    }
    p.m_tiles = (int)(m_pad / 256);
    p.k_blocks = (int)(k_pad / P_BK);
    p.k_blocks2 = (int)(k_pad2 / P_BK);
    const int tiles = p.m_tiles * p.n_tiles;
    const int pairs = tiles < info->pairs ? tiles : info->pairs;
    const dim3 grid(2 * pairs);
    CUtensorMap my = ma;  // unused unless the bulk-store epilogue runs
    if (!q_out && !chunk_dst && p.vec_ok && n % 128 == 0) {
      if (int rc = make_y_map(&my, y, n, rows_out, ldy)) return rc;
      p.tma_y = 1;
    }
    if (q_out && act == VDN_ACT_GELU_TANH)
      mxfp8_gemm_pair_kernel<EPI_QUANT_GELU><<<grid, THREADS, P_SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, sf, my, p);
    else if (q_out)
      mxfp8_gemm_pair_kernel<EPI_QUANT><<<grid, THREADS, P_SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, sf, my, p);
    else if (chunk_dst)
      mxfp8_gemm_pair_kernel<EPI_SCATTER><<<grid, THREADS, P_SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, sf, my, p);
    else
      mxfp8_gemm_pair_kernel<EPI_STORE><<<grid, THREADS, P_SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, sf, my, p);
    VDN_LAUNCH_CHECK("mxfp8 gemm (CTA pairs)");
    return VDN_OK;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < info->sms ? tiles : info->sms;
  if (q_out && act == VDN_ACT_GELU_TANH)
    mxfp8_gemm_kernel<EPI_QUANT_GELU><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, p);
  else if (q_out)
    mxfp8_gemm_kernel<EPI_QUANT><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, p);
  else if (chunk_dst)
    mxfp8_gemm_kernel<EPI_SCATTER><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, p);
  else
    mxfp8_gemm_kernel<EPI_STORE><<<grid, THREADS, SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, p);
  VDN_LAUNCH_CHECK("mxfp8 gemm");
  return VDN_OK;
}

extern "C" int vdn_mxfp8_gemm(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq,
                              const uint8_t* ws, const void* bias, int64_t m_pad, int64_t n,
                              int64_t n_pad, int64_t k_pad, int64_t rows_out, void* y, int64_t ldy,
                              int* status, cudaStream_t stream) {
  return launch_gemm(xq, xs, wq, ws, k_pad, nullptr, nullptr, nullptr, nullptr, 0, bias, m_pad, n,
                     n_pad, rows_out, y, ldy, nullptr, 0, nullptr, status, stream);
}

extern "C" int vdn_mxfp8_gemm_fused(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq,
                                    const uint8_t* ws, int64_t k_pad, const uint8_t* xq2,
                                    const uint8_t* xs2, const uint8_t* wq2, const uint8_t* ws2,
                                    int64_t k_pad2, const void* bias, int64_t m_pad, int64_t n,
                                    int64_t n_pad, int64_t rows_out, void* y, int64_t ldy,
                                    const void* resid, int64_t ldr, const void* gate, int* status,
                                    cudaStream_t stream) {
  return launch_gemm(xq, xs, wq, ws, k_pad, xq2, xs2, wq2, ws2, k_pad2, bias, m_pad, n, n_pad,
                     rows_out, y, ldy, resid, ldr, gate, status, stream);
}

extern "C" int vdn_mxfp8_gemm_scatter(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq,
                                      const uint8_t* ws, int64_t k_pad, const void* bias, int64_t m_pad,
                                      int64_t n, int64_t n_pad, int64_t rows_out,
                                      const uint64_t* chunk_dst, int64_t dst_ld, int64_t dst_row0,
                                      int* status, cudaStream_t stream) {
  if (!chunk_dst) return vdn::set_error(VDN_ERR_VALUE, "chunk_dst must not be null");
  return launch_gemm(xq, xs, wq, ws, k_pad, nullptr, nullptr, nullptr, nullptr, 0, bias, m_pad, n, n_pad,
                     rows_out, nullptr, 0, nullptr, 0, nullptr, status, stream, chunk_dst, dst_ld, dst_row0);
}

extern "C" int vdn_mxfp8_gemm_act_quantize(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq,
                                           const uint8_t* ws, int64_t k_pad, const void* bias,
                                           int64_t m_pad, int64_t n, int64_t n_pad, int64_t rows_out,
                                           int act, uint8_t* q, uint8_t* s, int* status,
                                           cudaStream_t stream) {
  if (act != VDN_ACT_GELU_TANH && act != 0)
    return vdn::set_error(VDN_ERR_VALUE, "act must be 0 (none) or VDN_ACT_GELU_TANH");
  if (!q || !s) return vdn::set_error(VDN_ERR_VALUE, "q and s must not be null");
  if (bias && !aligned16(bias)) return vdn::set_error(VDN_ERR_VALUE, "bias must be 16-byte aligned");
  return launch_gemm(xq, xs, wq, ws, k_pad, nullptr, nullptr, nullptr, nullptr, 0, bias, m_pad, n, n_pad,
                     rows_out, nullptr, 0, nullptr, 0, nullptr, status, stream, nullptr, 0, 0, act, q, s);
}
