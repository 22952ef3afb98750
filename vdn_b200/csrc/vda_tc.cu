// Tensor-core (tcgen05, kind::f16 bf16 -> fp32 in TMEM) VDA stages for d = 128.
//
// statistics  one CTA (256 threads) per (frame, head).  Raw k / v are streamed in
//             32-token chunks by TMA (4D tensor maps: d, token, head, frame; tokens
//             past S read as zero) into a 3-stage ring.  Eight threads per token
//             apply the features (SiLU, L2 over d, the eager bf16 rounding points)
//             and beta, and write four MN-major 128B-swizzled operands into one of
//             two operand buffers: kf, khi, klo = exact bf16 split of the fp32
//             product kf*beta (16 significant bits), vb = bf16(vf*beta).  One thread
//             then issues A += khi.kf^T + klo.kf^T and B += vb.kf^T (M = N = 128,
//             K = 16 tokens per MMA).  Epilogue: warps 0-3 read A, warps 4-7 read B
//             from TMEM; A is symmetrised through shared memory, B rounded to bf16.
// readout     one CTA (128 threads, two per SM) per (frame, head).  The gathered bf16
//             state [v][k] is the K-major B operand; 128-token q tiles arrive by TMA
//             (2 stages), each thread turns its row into features in place, and one
//             thread issues q.state^T (8 MMAs, K = 16) into one of two TMEM
//             accumulators.  The epilogue of the previous tile overlaps: thread =
//             TMEM lane = token, bf16 readout, RMSNorm over the row, * w, * gate,
//             token-major store.
// Reference: ec-jt/vdn src/models/linear_attention/scan.py:238-267 (statistics),
// branch.py:470-482 and ops/rms_norm.py:29-32 (readout and epilogue).
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace vdn {
namespace vtc {

using namespace sm100;

// Byte offset of 16-byte chunk c (0..7) of row `row` in a 128B-swizzled region.
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t c) {
  return row * 128u + ((c ^ (row & 7u)) << 4);
}

__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// ------------------------------------------------------------------ statistics
constexpr int ST_CH = 32;                       // tokens per chunk
constexpr int ST_RAW_STAGES = 3;
constexpr int ST_REGION = ST_CH * 128;          // 4 KB: 32 rows x 128 B
constexpr int ST_RAW_BYTES = 4 * ST_REGION;     // k r0, k r1, v r0, v r1
constexpr int ST_OP_BYTES = 8 * ST_REGION;      // kf, khi, klo, vb (2 regions each)
constexpr int ST_OPS = 2;
constexpr size_t ST_SMEM = 1024 + ST_RAW_STAGES * ST_RAW_BYTES + ST_OPS * ST_OP_BYTES + 128;

struct StatsParams {
  const uint16_t* beta;
  int64_t b_sf, b_ss, b_sh;
  float* A;
  float* B;
  int S, H;
  int* status;
};

template <bool FEATURES>
__global__ void __launch_bounds__(256, 2)
    stats_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const StatsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem;
  uint8_t* ops = raw + ST_RAW_STAGES * ST_RAW_BYTES;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(ops + ST_OPS * ST_OP_BYTES);
  uint64_t* mma_done = raw_full + ST_RAW_STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + ST_OPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int fh = blockIdx.x, f = fh / p.H, h = fh % p.H;
  const int nch = (p.S + ST_CH - 1) / ST_CH;

  if (tid == 0) {
    for (int s = 0; s < ST_RAW_STAGES; ++s) mbar_init(&raw_full[s], 1);
    for (int s = 0; s < ST_OPS; ++s) mbar_init(&mma_done[s], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_holder, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  auto issue_chunk = [&](int c) {
    uint8_t* st = raw + (c % ST_RAW_STAGES) * ST_RAW_BYTES;
    uint64_t* bar = &raw_full[c % ST_RAW_STAGES];
    mbar_arrive_expect_tx(bar, ST_RAW_BYTES);
    tma_load_4d(st, &tk, bar, 0, c * ST_CH, h, f);
    tma_load_4d(st + ST_REGION, &tk, bar, 64, c * ST_CH, h, f);
    tma_load_4d(st + 2 * ST_REGION, &tv, bar, 0, c * ST_CH, h, f);
    tma_load_4d(st + 3 * ST_REGION, &tv, bar, 64, c * ST_CH, h, f);
  };
  if (tid == 0)
    for (int c = 0; c < ST_RAW_STAGES && c < nch; ++c) issue_chunk(c);

  // Thread -> (token row in the chunk, 16 consecutive d): region r, chunks cc, cc+1.
  const uint32_t row = tid >> 3, e = tid & 7, r = e >> 2, cc = (e & 3) * 2;
  constexpr uint32_t kIdesc = idesc_bf16(128, 128, 1, 1);
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int rs = c % ST_RAW_STAGES, ob = c % ST_OPS;
    ok = __syncthreads_and(ok ? mbar_wait(&raw_full[rs], (c / ST_RAW_STAGES) & 1, abort_flag) : 0);
    if (!ok) break;
    if (c >= ST_OPS) {
      ok = __syncthreads_and(mbar_wait(&mma_done[ob], ((c - ST_OPS) / ST_OPS) & 1, abort_flag));
      if (!ok) break;
    }
    const uint8_t* st = raw + rs * ST_RAW_BYTES;
    uint8_t* op = ops + ob * ST_OP_BYTES;
    const int s = c * ST_CH + (int)row;
    float bt = 0.f;
    if (s < p.S) bt = bf16_bits_to_f32(p.beta[(int64_t)f * p.b_sf + (int64_t)s * p.b_ss + (int64_t)h * p.b_sh]);
    float kv[16], vv[16];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t off = r * ST_REGION + swz(row, cc + j);
      unpack8(*reinterpret_cast<const uint4*>(st + off), kv + 8 * j);
      unpack8(*reinterpret_cast<const uint4*>(st + 2 * ST_REGION + off), vv + 8 * j);
    }
    if (FEATURES) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        kv[i] = round_bf16(silu_fast(kv[i]));
        ss = fmaf(kv[i], kv[i], ss);
        vv[i] = round_bf16(silu_fast(vv[i]));
      }
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      ss += __shfl_xor_sync(0xffffffffu, ss, 4);
      const float nrm = fmaxf(round_bf16(sqrtf(ss)), round_bf16(1e-6f));
      const float inv = __fdiv_rn(1.0f, nrm);
#pragma unroll
      for (int i = 0; i < 16; ++i) kv[i] = round_bf16(kv[i] * inv);
    }
    float hi[16], lo[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float prod = kv[i] * bt;  // exact: two bf16 factors
      hi[i] = round_bf16(prod);
      lo[i] = round_bf16(prod - hi[i]);
      vv[i] = round_bf16(vv[i] * bt);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t off = r * ST_REGION + swz(row, cc + j);
      *reinterpret_cast<uint4*>(op + off) = pack8(kv + 8 * j);
      *reinterpret_cast<uint4*>(op + 2 * ST_REGION + off) = pack8(hi + 8 * j);
      *reinterpret_cast<uint4*>(op + 4 * ST_REGION + off) = pack8(lo + 8 * j);
      *reinterpret_cast<uint4*>(op + 6 * ST_REGION + off) = pack8(vv + 8 * j);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      if (c + ST_RAW_STAGES < nch) issue_chunk(c + ST_RAW_STAGES);  // raw stage rs is consumed
      const uint32_t base = smem_u32(op);
#pragma unroll
      for (int ks = 0; ks < ST_CH / 16; ++ks) {
        const uint32_t koff = ks * 16 * 128;  // 16 token rows
        const uint64_t dkf = desc_mn_sw128(base + koff, ST_REGION);
        const uint64_t dhi = desc_mn_sw128(base + 2 * ST_REGION + koff, ST_REGION);
        const uint64_t dlo = desc_mn_sw128(base + 4 * ST_REGION + koff, ST_REGION);
        const uint64_t dvb = desc_mn_sw128(base + 6 * ST_REGION + koff, ST_REGION);
        const uint32_t acc = (c | ks) != 0;
        mma_bf16(tmem, dhi, dkf, kIdesc, acc);
        mma_bf16(tmem, dlo, dkf, kIdesc, 1);
        mma_bf16(tmem + 128, dvb, dkf, kIdesc, acc);
      }
      tc_commit(&mma_done[ob]);
    }
  }
  // Wait for the last chunk's MMAs (they cover every earlier one).
  if (ok && nch > 0) {
    const int last = nch - 1;
    ok = __syncthreads_and(mbar_wait(&mma_done[last % ST_OPS], (last / ST_OPS) & 1, abort_flag));
  }
  tc_fence_after();
  if (ok) {
    // Epilogue: warps 0-3 hold A rows (lane quadrant = warp), warps 4-7 B rows.
    float* trans = reinterpret_cast<float*>(smem);  // [128][129], reuses the rings
    const int quad = warp & 3;
    const int mrow = quad * 32 + lane;
    const bool is_a = warp < 4;
    const uint32_t col0 = is_a ? 0 : 128;
    float* b_out = p.B + ((int64_t)fh * 128 + mrow) * 128;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(quad * 32) << 16) + col0 + cb * 32, v);
      tmem_ld_wait();
      if (is_a) {
#pragma unroll
        for (int i = 0; i < 32; ++i) trans[mrow * 129 + cb * 32 + i] = __uint_as_float(v[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(b_out + cb * 32 + i) =
              make_float4(round_bf16(__uint_as_float(v[i])), round_bf16(__uint_as_float(v[i + 1])),
                          round_bf16(__uint_as_float(v[i + 2])), round_bf16(__uint_as_float(v[i + 3])));
      }
    }
    __syncthreads();
    if (is_a) {
      float* a_out = p.A + ((int64_t)fh * 128 + mrow) * 128;
#pragma unroll 4
      for (int cidx = 0; cidx < 128; cidx += 4) {
        float4 o;
        o.x = 0.5f * (trans[mrow * 129 + cidx] + trans[cidx * 129 + mrow]);
        o.y = 0.5f * (trans[mrow * 129 + cidx + 1] + trans[(cidx + 1) * 129 + mrow]);
        o.z = 0.5f * (trans[mrow * 129 + cidx + 2] + trans[(cidx + 2) * 129 + mrow]);
        o.w = 0.5f * (trans[mrow * 129 + cidx + 3] + trans[(cidx + 3) * 129 + mrow]);
        *reinterpret_cast<float4*>(a_out + cidx) = o;
      }
    }
  } else {
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, 256);
  }
  if (tid == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}

// --------------------------------------------------------------------- readout
constexpr int RO_TOK = 128;
constexpr int RO_STAGES = 2;
constexpr int RO_TILE = 2 * RO_TOK * 128;       // 2 regions x 128 rows x 128 B = 32 KB
constexpr size_t RO_SMEM = 1024 + RO_TILE + RO_STAGES * RO_TILE + 128 * 4 + 128;

struct ReadoutParams {
  const uint16_t* gate;
  int64_t g_sf, g_ss, g_sh;
  const float* norm_w;
  float eps;
  uint16_t* out;
  int S, H;
  int* status;
};

__global__ void __launch_bounds__(128, 2)
    readout_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tstate,
                      const ReadoutParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* st_s = smem;
  uint8_t* q_s = smem + RO_TILE;
  float* w_s = reinterpret_cast<float*>(q_s + RO_STAGES * RO_TILE);
  uint64_t* state_full = reinterpret_cast<uint64_t*>(w_s + 128);
  uint64_t* q_full = state_full + 1;
  uint64_t* mma_done = q_full + RO_STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int fh = blockIdx.x, f = fh / p.H, h = fh % p.H;
  const int nt = (p.S + RO_TOK - 1) / RO_TOK;

  if (tid == 0) {
    mbar_init(state_full, 1);
    for (int s = 0; s < RO_STAGES; ++s) mbar_init(&q_full[s], 1);
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  w_s[tid] = round_bf16(p.norm_w[tid]);
  if (warp == 0) tmem_alloc(tmem_holder, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  auto issue_tile = [&](int i) {
    uint8_t* dst = q_s + (i % RO_STAGES) * RO_TILE;
    uint64_t* bar = &q_full[i % RO_STAGES];
    mbar_arrive_expect_tx(bar, RO_TILE);
    tma_load_4d(dst, &tq, bar, 0, i * RO_TOK, h, f);
    tma_load_4d(dst + RO_TILE / 2, &tq, bar, 64, i * RO_TOK, h, f);
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(state_full, RO_TILE);
    tma_load_2d(st_s, &tstate, state_full, 0, fh * 128);
    tma_load_2d(st_s + RO_TILE / 2, &tstate, state_full, 64, fh * 128);
    for (int i = 0; i < RO_STAGES && i < nt; ++i) issue_tile(i);
  }
  constexpr uint32_t kIdesc = idesc_bf16(128, 128, 0, 0);
  const uint32_t t = tid;
  bool ok = true;

  auto epilogue = [&](int j) -> bool {
    const int b = j & 1;
    if (!__syncthreads_and(mbar_wait(&mma_done[b], (j >> 1) & 1, abort_flag))) return false;
    tc_fence_after();
    if (tid == 0 && j + RO_STAGES < nt) issue_tile(j + RO_STAGES);  // its q stage is free now
    const int s = j * RO_TOK + (int)t;
    const bool valid = s < p.S;
    const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + b * 128;
    float ss = 0.f;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + cb * 32, v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float x = round_bf16(__uint_as_float(v[i]));
        ss = fmaf(x, x, ss);
      }
    }
    const float nrm = sqrtf(ss);
    const float inv = round_bf16(__fdiv_rn(1.0f, sqrtf(nrm * nrm / 128.0f + p.eps)));
    const uint16_t* grow = p.gate + (int64_t)f * p.g_sf + (int64_t)s * p.g_ss + (int64_t)h * p.g_sh;
    uint16_t* orow = p.out + ((int64_t)f * p.S + s) * ((int64_t)p.H * 128) + (int64_t)h * 128;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(taddr + cb * 32, v);
      tmem_ld_wait();
      if (!valid) continue;
      float g[32], y[32];
#pragma unroll
      for (int i = 0; i < 4; ++i) unpack8(*reinterpret_cast<const uint4*>(grow + cb * 32 + 8 * i), g + 8 * i);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float rr = round_bf16(__uint_as_float(v[i]));
        const float yy = round_bf16(round_bf16(rr * inv) * w_s[cb * 32 + i]);
        y[i] = yy * g[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(orow + cb * 32 + 8 * i) = pack8(y + 8 * i);
    }
    tc_fence_before();
    return true;
  };

  for (int i = 0; i < nt && ok; ++i) {
    const int qs = i % RO_STAGES;
    ok = __syncthreads_and(mbar_wait(&q_full[qs], (i / RO_STAGES) & 1, abort_flag));
    if (!ok) break;
    // Row t of the tile -> features in place (SiLU, L2 over d, eager rounding).
    uint8_t* tile = q_s + qs * RO_TILE;
    uint32_t packed[64];
    float ssum = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint32_t off = (c >> 3) * (RO_TILE / 2) + swz(t, c & 7);
      float x[8];
      unpack8(*reinterpret_cast<const uint4*>(tile + off), x);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        x[k] = round_bf16(silu_fast(x[k]));
        ssum = fmaf(x[k], x[k], ssum);
      }
      const uint4 pk = pack8(x);
      packed[4 * c] = pk.x;
      packed[4 * c + 1] = pk.y;
      packed[4 * c + 2] = pk.z;
      packed[4 * c + 3] = pk.w;
    }
    const float nrm = fmaxf(round_bf16(sqrtf(ssum)), round_bf16(1e-6f));
    const float inv = __fdiv_rn(1.0f, nrm);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      float x[8];
      unpack8(make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]), x);
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = round_bf16(x[k] * inv);
      const uint32_t off = (c >> 3) * (RO_TILE / 2) + swz(t, c & 7);
      *reinterpret_cast<uint4*>(tile + off) = pack8(x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      if (i == 0 && !mbar_wait(state_full, 0, abort_flag)) {
        ok = false;
      } else {
        const uint32_t qa = smem_u32(tile), sb = smem_u32(st_s);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * (RO_TILE / 2) + (ks & 3) * 32;
          mma_bf16(tmem + (i & 1) * 128, desc_k_sw128(qa + off), desc_k_sw128(sb + off), kIdesc, ks > 0);
        }
        tc_commit(&mma_done[i & 1]);
      }
    }
    ok = __syncthreads_and(ok && !*abort_flag);
    if (!ok) break;
    if (i >= 1 && !epilogue(i - 1)) {
      ok = false;
      break;
    }
  }
  if (ok && nt > 0) epilogue(nt - 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, 256);
  }
  if (tid == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}

// ------------------------------------------------------------------- host side
static bool is16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// 4D bf16 map over (d = 128, token, head, frame) with element strides ss, sh, sf.
static int map_tokens(CUtensorMap* m, const void* base, int64_t sf, int64_t ss, int64_t sh, int F,
                      int S, int H, int box_tokens) {
  cuuint64_t dims[4] = {128, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)F};
  cuuint64_t strides[3] = {(cuuint64_t)(ss * 2), (cuuint64_t)(sh * 2), (cuuint64_t)(sf * 2)};
  cuuint32_t box[4] = {64, (cuuint32_t)box_tokens, 1, 1};
  return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box);
}

static bool strides_ok(const void* p, int64_t sf, int64_t ss, int64_t sh) {
  return is16(p) && sf > 0 && ss > 0 && sh > 0 && sf % 8 == 0 && ss % 8 == 0 && sh % 8 == 0;
}

}  // namespace vtc

bool tc_stats_supported(int d, const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh, const void* v,
                        int64_t v_sf, int64_t v_ss, int64_t v_sh) {
  return d == 128 && vtc::strides_ok(k, k_sf, k_ss, k_sh) && vtc::strides_ok(v, v_sf, v_ss, v_sh);
}

int launch_stats_tc(const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sf,
                    int64_t v_ss, int64_t v_sh, const void* beta, int64_t b_sf, int64_t b_ss,
                    int64_t b_sh, int features_applied, int F, int S, int H, float* A, float* B,
                    int* status, cudaStream_t stream) {
  using namespace vtc;
  CUtensorMap mk, mv;
  if (int rc = map_tokens(&mk, k, k_sf, k_ss, k_sh, F, S, H, ST_CH)) return rc;
  if (int rc = map_tokens(&mv, v, v_sf, v_ss, v_sh, F, S, H, ST_CH)) return rc;
  StatsParams p{static_cast<const uint16_t*>(beta), b_sf, b_ss, b_sh, A, B, S, H, status};
  static bool attr_set[2] = {false, false};
  if (features_applied) {
    if (!attr_set[0]) {
      VDN_CUDA_TRY(cudaFuncSetAttribute(stats_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ST_SMEM));
      attr_set[0] = true;
    }
    stats_tc_kernel<false><<<F * H, 256, ST_SMEM, stream>>>(mk, mv, p);
  } else {
    if (!attr_set[1]) {
      VDN_CUDA_TRY(cudaFuncSetAttribute(stats_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ST_SMEM));
      attr_set[1] = true;
    }
    stats_tc_kernel<true><<<F * H, 256, ST_SMEM, stream>>>(mk, mv, p);
  }
  VDN_LAUNCH_CHECK("vda statistics (tcgen05)");
  return VDN_OK;
}

bool tc_readout_supported(int d, const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh,
                          const void* state, const void* gate, int64_t g_ss, int64_t g_sh) {
  return d == 128 && vtc::strides_ok(q, q_sf, q_ss, q_sh) && vtc::is16(state) && vtc::is16(gate) &&
         g_ss % 8 == 0 && g_sh % 8 == 0;
}

int launch_readout_tc(const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh, const void* state,
                      const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh, const float* norm_w,
                      float eps, int F, int S, int H, void* out, int* status, cudaStream_t stream) {
  using namespace vtc;
  CUtensorMap mq, ms;
  if (int rc = map_tokens(&mq, q, q_sf, q_ss, q_sh, F, S, H, RO_TOK)) return rc;
  cuuint64_t dims[2] = {128, (cuuint64_t)F * H * 128};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, 128};
  if (int rc = encode_map(&ms, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, state, dims, strides, box)) return rc;
  ReadoutParams p{static_cast<const uint16_t*>(gate), g_sf, g_ss, g_sh, norm_w, eps,
                  static_cast<uint16_t*>(out), S, H, status};
  static bool attr_set = false;
  if (!attr_set) {
    VDN_CUDA_TRY(cudaFuncSetAttribute(readout_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RO_SMEM));
    attr_set = true;
  }
  readout_tc_kernel<<<F * H, 128, RO_SMEM, stream>>>(mq, ms, p);
  VDN_LAUNCH_CHECK("vda readout (tcgen05)");
  return VDN_OK;
}

}  // namespace vdn
