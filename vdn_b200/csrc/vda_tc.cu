// Tensor-core (tcgen05, kind::f16 bf16 -> fp32 in TMEM) VDA stages for d = 128.
//
// statistics  persistent, one CTA per SM walking (frame, head) items.  Raw k / v
//             are streamed in 32-token chunks by TMA (4D tensor maps: d, token,
//             head, frame; tokens past S read as zero) into a ring of stages.
//             Sixteen threads per token apply the features (SiLU, L2 over d, the
//             eager bf16 rounding points) and beta, and write four MN-major
//             128B-swizzled operands in place: kf, khi + klo = the exact bf16 split
//             of the fp32 product kf*beta (16 significant bits), vb = bf16(vf*beta).
//             One thread then issues A2 += khi.kf^T + klo.kf^T + kf.khi^T + kf.klo^T
//             (twice the symmetrised A, accumulated on the tensor cores) and
//             B += vb.kf^T (M = N = 128, K = 16 tokens per MMA).  Epilogue: A = A2 / 2
//             and B rounded to bf16, straight from TMEM.
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

// Named-barrier AND vote over `count` threads: every participant gets the same
// answer, so a group of warps leaves a loop together (a warp that left alone
// would strand the others at the group's next barrier).
__device__ __forceinline__ bool bar_and(uint32_t id, uint32_t count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// bf16 pair helpers: unpack a packed pair, and the round-to-nearest product of two
// bf16 pairs (exact product, one rounding: the bf16 multiply of the eager body).
__device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xFFFF0000u);
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// SiLU inputs arrive as packed bf16 pairs; values below -43.5 (bf16 0xC22E) are raised
// to it, where |silu(x)| < 6e-18 (compare the unsigned 16-bit patterns: every negative
// value below -43.5, -inf included, has a larger pattern than 0xC22E, every positive
// value a smaller one).  This bounds 1 + e^-x by 8e18 for silu_pair.
__device__ __forceinline__ uint32_t clamp_silu_in(uint32_t w) { return __vminu2(w, 0xC22EC22Eu); }

// x * sigmoid(x) for two values clamped by clamp_silu_in: x0 / a and x1 / b with
// a = 1 + 2^(-x0 log2 e), b likewise, both reciprocals from one MUFU reciprocal of
// a * b (< 2^126: 1/a = b / (a b)); the products run as f32x2 pairs.  The transforms
// that use it are bound by issue slots and the MUFU pipe together (a Newton reciprocal
// on the FMA pipe, or the pair trick in scalar arithmetic, measured slower): this form
// takes three MUFU operations and five issue slots of arithmetic for the pair.
__device__ __forceinline__ void silu_pair(float& x0, float& x1) {
  const f2 xx = f2_pack(x0, x1);
  float e0, e1;
  f2_unpack(f2_mul(xx, f2_pack(-1.4426950408889634f, -1.4426950408889634f)), e0, e1);
  float a, b;
  f2_unpack(f2_add(f2_pack(ex2_approx(e0), ex2_approx(e1)), f2_pack(1.0f, 1.0f)), a, b);
  const float r = rcp_approx(a * b);
  f2_unpack(f2_mul(xx, f2_mul(f2_pack(b, a), f2_pack(r, r))), x0, x1);
}

// ------------------------------------------------------------------ statistics
// Persistent, warp-specialised: grid = min(F*H, SMs), one CTA per SM walking
// (frame, head) items.  Warp 0 lane 0 streams 32-token raw k / v chunks by TMA
// into a 6-stage ring; warps 2-17 (16 threads per token, one 8-element chunk of
// k and of v each) apply features and beta and write kf / vb in place plus the
// khi / klo split; warp 1 lane 0 issues A2 += khi.kf^T + klo.kf^T + kf.khi^T +
// kf.klo^T and B += vb.kf^T into one of two TMEM accumulator pairs (512 columns);
// warps 18-21 drain an item's A = A2 / 2 and B (bf16-rounded) while the next item
// streams, in whole-line stores after an in-warp transpose (row-per-thread stores, 32
// rows per instruction, held up the transform warps' shared-memory traffic for ~6k
// cycles at every item boundary).  A stage is held from its TMA load until its MMAs complete, and the
// load alone takes ~3.2k cycles, so the ring depth sets the chunk rate: the
// symmetrisation moved onto the tensor cores to free the 66 KB transpose buffer
// for two more stages.
constexpr int ST_CH = 32;                       // tokens per chunk
constexpr int ST_STAGES = 6;
constexpr int ST_REGION = ST_CH * 128;          // 4 KB: 32 rows x 128 B
constexpr int ST_STAGE_BYTES = 8 * ST_REGION;   // k(kf), v(vb), khi, klo: 2 regions each
constexpr int ST_RAW_BYTES = 4 * ST_REGION;     // what TMA writes per stage
constexpr int ST_THREADS = 736;             // 2 + 16 transform + 4 epilogue + 1 beta warps
constexpr int ST_NBAR = 3 * ST_STAGES + 2 * 2 + 1;
constexpr size_t ST_SMEM = 1024 + ST_STAGES * ST_STAGE_BYTES + ST_STAGES * ST_CH * 4 + ST_NBAR * 8 + 64;
static_assert(ST_SMEM <= 232448, "shared memory per CTA");

struct StatsParams {
  const uint16_t* beta;
  int64_t b_sf, b_ss, b_sh;
  float* A;
  float* B;                // fp32 [items][128][128], or bf16 when b_bf16 (its values are bf16 either way)
  int b_bf16;
  int S, H, items;
  int* status;
};

template <bool FEATURES>
__global__ void __launch_bounds__(ST_THREADS, 1)
    stats_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const StatsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* beta_s = reinterpret_cast<float*>(smem + ST_STAGES * ST_STAGE_BYTES);  // [stage][token]
  uint64_t* bars = reinterpret_cast<uint64_t*>(beta_s + ST_STAGES * ST_CH);
  uint64_t* full = bars;
  uint64_t* ready = full + ST_STAGES;
  uint64_t* empty = ready + ST_STAGES;
  uint64_t* acc_full = empty + ST_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nch = (p.S + ST_CH - 1) / ST_CH;

  if (tid == 0) {
    for (int s = 0; s < ST_STAGES; ++s) {
      mbar_init(&full[s], 2);    // the producer (with the TMA bytes) and the beta warp
      mbar_init(&ready[s], 16);  // one arrival per transform warp
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int g = 0;
      uint32_t pend = 0, pend_phase = 0;
      for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x) {
        const int f = item / p.H, h = item % p.H;
        for (int c = 0; c < nch; ++c, ++g) {
          const int s = g % ST_STAGES;
          const uint32_t ph = (g / ST_STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) break;
          uint8_t* st = stages + s * ST_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], ST_RAW_BYTES);
          tma_load_4d(st, &tk, &full[s], 0, c * ST_CH, h, f);
          tma_load_4d(st + ST_REGION, &tk, &full[s], 64, c * ST_CH, h, f);
          tma_load_4d(st + 2 * ST_REGION, &tv, &full[s], 0, c * ST_CH, h, f);
          tma_load_4d(st + 3 * ST_REGION, &tv, &full[s], 64, c * ST_CH, h, f);
          pend |= 1u << s;
          pend_phase = (pend_phase & ~(1u << s)) | (ph << s);
        }
      }
      if (*abort_flag) {
        for (int s = 0; s < ST_STAGES; ++s) {
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
      constexpr uint32_t kIdesc = idesc_bf16(128, 128, 1, 1);
      int g = 0, k = 0;
      bool issued = false;
      for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x, ++k) {
        const int b = k & 1;
        if (!mbar_wait(&acc_empty[b], ((k >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t acc_a = tmem + b * 256, acc_b = acc_a + 128;
        bool ok = true;
        for (int c = 0; c < nch; ++c, ++g) {
          const int s = g % ST_STAGES;
          if (!mbar_wait(&ready[s], (g / ST_STAGES) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(stages + s * ST_STAGE_BYTES);
#pragma unroll
          for (int ks = 0; ks < ST_CH / 16; ++ks) {
            const uint32_t koff = ks * 16 * 128;  // 16 token rows
            const uint64_t dkf = desc_mn_sw128(base + koff, ST_REGION);
            const uint64_t dvb = desc_mn_sw128(base + 2 * ST_REGION + koff, ST_REGION);
            const uint64_t dhi = desc_mn_sw128(base + 4 * ST_REGION + koff, ST_REGION);
            const uint64_t dlo = desc_mn_sw128(base + 6 * ST_REGION + koff, ST_REGION);
            const uint32_t acc = (c | ks) != 0;
            mma_bf16(acc_a, dhi, dkf, kIdesc, acc);
            mma_bf16(acc_a, dlo, dkf, kIdesc, 1);
            mma_bf16(acc_a, dkf, dhi, kIdesc, 1);
            mma_bf16(acc_a, dkf, dlo, kIdesc, 1);
            mma_bf16(acc_b, dvb, dkf, kIdesc, acc);
          }
          issued = true;
          tc_commit(&empty[s]);
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
  } else if (warp < 18) {
    // ----------------------------------------------------------- transform
    const uint32_t t = tid - 64;                 // 0..511
    const uint32_t row = t >> 4, e = t & 15, r = e >> 3, cc = e & 7;
    int g = 0;
    for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x) {
      // One chunk: features, beta and the khi / klo split, in place in its stage.
      // Returns false when a wait gave up.
      auto chunk = [&]() -> bool {
        const int s = g % ST_STAGES;
        // Warp-uniform outcome: the warp's lanes meet again at the __syncwarp below.
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (g / ST_STAGES) & 1, abort_flag))) {
          return false;
        }
        uint8_t* st = stages + s * ST_STAGE_BYTES;
        const float bt = beta_s[s * ST_CH + row];
        const uint32_t off = r * ST_REGION + swz(row, cc);
        const uint4 kin = *reinterpret_cast<const uint4*>(st + off);
        const uint4 vin = *reinterpret_cast<const uint4*>(st + 2 * ST_REGION + off);
        uint32_t kfw[4] = {kin.x, kin.y, kin.z, kin.w};   // kf as packed bf16 pairs
        uint32_t vsw[4] = {vin.x, vin.y, vin.z, vin.w};   // bf16(silu(v)) (or v) pairs
        float kv[8];
        // Features in f32x2 pairs: bf16(silu), the L2 norm (its square root and
        // reciprocal approximate, within fp32 ulps of the exact ones and then rounded
        // to bf16 or applied before a bf16 rounding), bf16(x / norm); each bf16 result
        // stays packed as the conversion writes it and is unpacked only where fp32
        // arithmetic needs it.
        if (FEATURES) {
          f2 ss2 = f2_pack(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float a, b;
            unpack2(clamp_silu_in(kfw[i]), a, b);
            silu_pair(a, b);
            kfw[i] = pack_bf16x2(a, b);
            unpack2(kfw[i], kv[2 * i], kv[2 * i + 1]);
            const f2 k2 = f2_pack(kv[2 * i], kv[2 * i + 1]);
            ss2 = f2_fma(k2, k2, ss2);
            unpack2(clamp_silu_in(vsw[i]), a, b);
            silu_pair(a, b);
            vsw[i] = pack_bf16x2(a, b);
          }
          float s0, s1;
          f2_unpack(ss2, s0, s1);
          float ss = s0 + s1;
          ss += __shfl_xor_sync(0xffffffffu, ss, 1);
          ss += __shfl_xor_sync(0xffffffffu, ss, 2);
          ss += __shfl_xor_sync(0xffffffffu, ss, 4);
          ss += __shfl_xor_sync(0xffffffffu, ss, 8);
          const float nrm = fmaxf(round_bf16(sqrt_approx(ss)), round_bf16(1e-6f));
          const float inv = rcp_approx(nrm);
          const f2 inv2 = f2_pack(inv, inv);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float a, b;
            f2_unpack(f2_mul(f2_pack(kv[2 * i], kv[2 * i + 1]), inv2), a, b);
            kfw[i] = pack_bf16x2(a, b);
            unpack2(kfw[i], kv[2 * i], kv[2 * i + 1]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) unpack2(kfw[i], kv[2 * i], kv[2 * i + 1]);
        }
        // kf * beta is exact in fp32 (two bf16 factors, 16 significant bits): its upper
        // half (bf16 truncation, hi) and the residual (itself a bf16 value) split it.
        // vb = bf16(v * beta) is one bf16 pair multiply (exact product, one rounding).
        uint32_t hi2[4], lo2[4], vb2[4];
        const f2 bt2 = f2_pack(bt, bt), m1 = f2_pack(-1.f, -1.f);
        const uint32_t bb = __float_as_uint(bt) >> 16, btb = bb | (bb << 16);   // (beta, beta) bf16x2
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const f2 p2 = f2_mul(f2_pack(kv[2 * i], kv[2 * i + 1]), bt2);
          float p0, p1;
          f2_unpack(p2, p0, p1);
          const float h0 = __uint_as_float(__float_as_uint(p0) & 0xFFFF0000u);
          const float h1 = __uint_as_float(__float_as_uint(p1) & 0xFFFF0000u);
          hi2[i] = pack_exact2(p0, p1);
          float l0, l1;
          f2_unpack(f2_fma(f2_pack(h0, h1), m1, p2), l0, l1);
          lo2[i] = pack_exact2(l0, l1);
          vb2[i] = mul_bf16x2(vsw[i], btb);
        }
        *reinterpret_cast<uint4*>(st + off) = make_uint4(kfw[0], kfw[1], kfw[2], kfw[3]);
        *reinterpret_cast<uint4*>(st + 2 * ST_REGION + off) = make_uint4(vb2[0], vb2[1], vb2[2], vb2[3]);
        *reinterpret_cast<uint4*>(st + 4 * ST_REGION + off) = make_uint4(hi2[0], hi2[1], hi2[2], hi2[3]);
        *reinterpret_cast<uint4*>(st + 6 * ST_REGION + off) = make_uint4(lo2[0], lo2[1], lo2[2], lo2[3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[s]);
        ++g;
        return true;
      };
      bool ok = true;
      for (int c = 0; c < nch && ok; ++c) ok = chunk();
      if (!ok) break;
    }
  } else if (warp == 22) {
    // ---------------------------------------------------------------- beta
    // One lane per token: beta of a stage's 32 tokens into shared memory as soon as
    // the stage is free (alongside the producer's k / v copies), then one arrival on
    // the stage's full barrier.  The transform warps read it from there, so no global
    // load sits in their loop.
    int g = 0;
    for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x) {
      const int f = item / p.H, h = item % p.H;
      const uint16_t* bcol = p.beta + (int64_t)f * p.b_sf + (int64_t)h * p.b_sh;
      bool ok = true;
      for (int c = 0; c < nch; ++c, ++g) {
        const int s = g % ST_STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ((g / ST_STAGES) & 1) ^ 1, abort_flag))) {
          ok = false;
          break;
        }
        const int tok = c * ST_CH + lane;
        beta_s[s * ST_CH + lane] = tok < p.S ? bf16_bits_to_f32(bcol[(int64_t)tok * p.b_ss]) : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;                   // warps 18..21 -> quadrants 2,3,0,1
    int k = 0;
    for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x, ++k) {
      const int b = k & 1;
      if (!bar_and(1, 128, mbar_wait(&acc_full[b], (k >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + b * 256;
      // This warp's 32 rows of the item's A and B; each 32-column block leaves through
      // an in-warp transpose as whole-line stores.
      const int64_t row0 = (int64_t)item * 128 + quad * 32;
      uint32_t* a_out = reinterpret_cast<uint32_t*>(p.A + row0 * 128);
      uint32_t* b_out = reinterpret_cast<uint32_t*>(p.B) + row0 * (p.b_bf16 ? 64 : 128);
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t va[32], vb[32];
        tmem_ld_32x32b_x32(lane_base + cb * 32, va);
        tmem_ld_32x32b_x32(lane_base + 128 + cb * 32, vb);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) va[i] = __float_as_uint(0.5f * __uint_as_float(va[i]));
        store_warp_rows_32x32(a_out + cb * 32, 128, va, lane);
        if (p.b_bf16) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1]));
          store_warp_rows_32x16(b_out + cb * 16, 64, w, lane);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) vb[i] = __float_as_uint(round_bf16(__uint_as_float(vb[i])));
          store_warp_rows_32x32(b_out + cb * 32, 128, vb, lane);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);                 // TMEM pair b may be refilled
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
  if (tid == 0 && *abort_flag && p.status) atomicExch(p.status, VDN_ERR_TIMEOUT);
}

// --------------------------------------------------------------------- readout
// Persistent, warp-specialised: grid = min(F*H, SMs), one CTA per SM walking
// (frame, head) items.  Warp 0 lane 0 streams the item's bf16 state (double
// buffered), its 128-token q tiles (2-stage ring) and the matching gate tiles
// (3-stage ring) by TMA; warps 2-9 turn the q tile into features in place (two
// threads per token row, 64 columns each: measured 10% faster than four warps);
// warp 1 lane 0 issues q.state^T into one of two TMEM accumulators; warps 10-13
// drain them (thread = TMEM lane = token): bf16 readout, RMSNorm over the row, * w,
// * the gate row read from the staged gate tile.  The result overwrites the gate in
// shared memory and leaves by one TMA store per 64-column half, so global memory
// sees only bulk tensor copies (a row-per-thread epilogue touches 32 rows per load
// or store instruction).  Hand-offs are mbarriers; every wait is bounded.
constexpr int RO_TOK = 128;
constexpr int RO_STAGES = 2;                    // q tiles
constexpr int RO_GSTAGES = 3;                   // gate / output tiles
constexpr int RO_THREADS = 448;
constexpr int RO_TILE = 2 * RO_TOK * 128;       // 2 regions x 128 rows x 128 B = 32 KB
constexpr int RO_NBAR = 3 * RO_STAGES + 2 * RO_GSTAGES + 2 * 2 + 2 * 2 + 1;
constexpr size_t RO_SMEM =
    1024 + 2 * RO_TILE + (RO_STAGES + RO_GSTAGES) * RO_TILE + 128 * 4 + RO_NBAR * 8 + 64;
static_assert(RO_SMEM <= 232448, "shared memory per CTA");

struct ReadoutParams {
  const float* norm_w;
  float eps;
  int S, H, items;
  int* status;
};

__global__ void __launch_bounds__(RO_THREADS, 1)
    readout_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tstate,
                      const __grid_constant__ CUtensorMap tgate, const __grid_constant__ CUtensorMap tout,
                      const ReadoutParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* st_s = smem;                           // 2 state buffers
  uint8_t* q_s = smem + 2 * RO_TILE;              // RO_STAGES q tiles
  uint8_t* g_s = q_s + RO_STAGES * RO_TILE;       // RO_GSTAGES gate / output tiles
  float* w_s = reinterpret_cast<float*>(g_s + RO_GSTAGES * RO_TILE);
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_s + 128);
  uint64_t* q_full = bars;
  uint64_t* q_ready = q_full + RO_STAGES;
  uint64_t* q_empty = q_ready + RO_STAGES;
  uint64_t* g_full = q_empty + RO_STAGES;
  uint64_t* g_empty = g_full + RO_GSTAGES;
  uint64_t* acc_full = g_empty + RO_GSTAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* st_full = acc_empty + 2;
  uint64_t* st_empty = st_full + 2;
  uint64_t* mma_drain = st_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nt = (p.S + RO_TOK - 1) / RO_TOK;

  if (tid == 0) {
    for (int s = 0; s < RO_STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_ready[s], 8);  // one arrival per transform warp
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < RO_GSTAGES; ++s) {
      mbar_init(&g_full[s], 1);
      mbar_init(&g_empty[s], 1);  // the store issuer, once the tile's store has read it
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
      mbar_init(&st_full[b], 1);
      mbar_init(&st_empty[b], 1);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (tid < 128) w_s[tid] = round_bf16(p.norm_w[tid]);
  if (warp == 1) tmem_alloc(tmem_holder, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int g = 0, k = 0;
      uint32_t pend = 0, pend_phase = 0, gpend = 0, gpend_phase = 0;
      for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x, ++k) {
        const int f = item / p.H, h = item % p.H, sb = k & 1;
        if (!mbar_wait(&st_empty[sb], ((k >> 1) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&st_full[sb], RO_TILE);
        tma_load_2d(st_s + sb * RO_TILE, &tstate, &st_full[sb], 0, item * 128);
        tma_load_2d(st_s + sb * RO_TILE + RO_TILE / 2, &tstate, &st_full[sb], 64, item * 128);
        for (int i = 0; i < nt; ++i, ++g) {
          const int s = g % RO_STAGES, gs = g % RO_GSTAGES;
          const uint32_t ph = (g / RO_STAGES) & 1, gph = (g / RO_GSTAGES) & 1;
          if (!mbar_wait(&q_empty[s], ph ^ 1, abort_flag)) break;
          uint8_t* dst = q_s + s * RO_TILE;
          mbar_arrive_expect_tx(&q_full[s], RO_TILE);
          tma_load_4d(dst, &tq, &q_full[s], 0, i * RO_TOK, h, f);
          tma_load_4d(dst + RO_TILE / 2, &tq, &q_full[s], 64, i * RO_TOK, h, f);
          pend |= 1u << s;
          pend_phase = (pend_phase & ~(1u << s)) | (ph << s);
          if (!mbar_wait(&g_empty[gs], gph ^ 1, abort_flag)) break;
          uint8_t* gdst = g_s + gs * RO_TILE;
          mbar_arrive_expect_tx(&g_full[gs], RO_TILE);
          tma_load_4d(gdst, &tgate, &g_full[gs], 0, i * RO_TOK, h, f);
          tma_load_4d(gdst + RO_TILE / 2, &tgate, &g_full[gs], 64, i * RO_TOK, h, f);
          gpend |= 1u << gs;
          gpend_phase = (gpend_phase & ~(1u << gs)) | (gph << gs);
        }
      }
      if (*abort_flag) {  // let every issued copy land before the CTA may exit
        for (int s = 0; s < RO_STAGES; ++s) {
          if (!(pend >> s & 1)) continue;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&q_full[s], (pend_phase >> s) & 1) && globaltimer() - t0 < kWaitLimitNs) {
          }
        }
        for (int s = 0; s < RO_GSTAGES; ++s) {
          if (!(gpend >> s & 1)) continue;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&g_full[s], (gpend_phase >> s) & 1) && globaltimer() - t0 < kWaitLimitNs) {
          }
        }
        for (int b = 0; b < 2 && k > b; ++b) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&st_full[(k - 1 - b) & 1], (((k - 1 - b) >> 1) & 1)) &&
                 globaltimer() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ----------------------------------------------------------------- MMA
      constexpr uint32_t kIdesc = idesc_bf16(128, 128, 0, 0);
      int g = 0, k = 0;
      bool issued = false;
      for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x, ++k) {
        const int sb = k & 1;
        if (!mbar_wait(&st_full[sb], (k >> 1) & 1, abort_flag)) break;
        const uint32_t sbase = smem_u32(st_s + sb * RO_TILE);
        bool ok = true;
        for (int i = 0; i < nt; ++i, ++g) {
          const int s = g % RO_STAGES, b = g & 1;
          if (!mbar_wait(&q_ready[s], (g / RO_STAGES) & 1, abort_flag) ||
              !mbar_wait(&acc_empty[b], ((g >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qa = smem_u32(q_s + s * RO_TILE);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t off = (ks >> 2) * (RO_TILE / 2) + (ks & 3) * 32;
            mma_bf16(tmem + b * 128, desc_k_sw128(qa + off), desc_k_sw128(sbase + off), kIdesc, ks > 0);
          }
          issued = true;
          tc_commit(&q_empty[s]);
          tc_commit(&acc_full[b]);
        }
        if (!ok) break;
        tc_commit(&st_empty[sb]);
      }
      if (*abort_flag && issued) {
        // The MMAs already issued must finish before TMEM is freed.
        tc_commit(mma_drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(mma_drain, 0) && globaltimer() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp < 10) {
    // ----------------------------------------------------------- transform
    const uint32_t t = tid - 64;                 // 0..255
    const uint32_t row = t >> 1, half = t & 1;   // lanes 2k, 2k+1 share a token row
    int g = 0;
    for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x) {
      bool ok = true;
      for (int i = 0; i < nt; ++i, ++g) {
        const int s = g % RO_STAGES;
        // Warp-uniform outcome: the warp's lanes meet again at the __syncwarp below.
        if (!__all_sync(0xffffffffu, mbar_wait(&q_full[s], (g / RO_STAGES) & 1, abort_flag))) {
          ok = false;
          break;
        }
        uint8_t* region = q_s + s * RO_TILE + half * (RO_TILE / 2);
        // Pass 1: bf16(silu) written back in place, sum of squares; pass 2: / norm.
        f2 ss2 = f2_pack(0.f, 0.f);
#pragma unroll 4
        for (int c = 0; c < 8; ++c) {
          uint4* ptr = reinterpret_cast<uint4*>(region + swz(row, c));
          const uint4 w4 = *ptr;
          uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float a, b;
            unpack2(clamp_silu_in(ww[i]), a, b);
            silu_pair(a, b);
            ww[i] = pack_bf16x2(a, b);
            unpack2(ww[i], a, b);
            const f2 x2 = f2_pack(a, b);
            ss2 = f2_fma(x2, x2, ss2);
          }
          *ptr = make_uint4(ww[0], ww[1], ww[2], ww[3]);
        }
        float s0, s1;
        f2_unpack(ss2, s0, s1);
        float ssum = s0 + s1;
        ssum += __shfl_xor_sync(0xffffffffu, ssum, 1);
        const float nrm = fmaxf(round_bf16(sqrt_approx(ssum)), round_bf16(1e-6f));
        const float inv = rcp_approx(nrm);
#pragma unroll 4
        for (int c = 0; c < 8; ++c) {
          uint4* ptr = reinterpret_cast<uint4*>(region + swz(row, c));
          float x[8];
          unpack8(*ptr, x);
#pragma unroll
          for (int kk = 0; kk < 8; kk += 2) f2_unpack(f2_mul(f2_pack(x[kk], x[kk + 1]), f2_pack(inv, inv)), x[kk], x[kk + 1]);
          *ptr = pack8(x);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_ready[s]);
      }
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;                   // warps 10..13
    const uint32_t erow = quad * 32 + lane;
    const bool issuer = warp == 10 && lane == 0;
    int g = 0;
    for (int item = blockIdx.x; item < p.items && !*abort_flag; item += gridDim.x) {
      const int f = item / p.H, h = item % p.H;
      bool ok = true;
      for (int i = 0; i < nt; ++i, ++g) {
        const int b = g & 1, gs = g % RO_GSTAGES;
        const bool got = mbar_wait(&g_full[gs], (g / RO_GSTAGES) & 1, abort_flag) &&
                         mbar_wait(&acc_full[b], (g >> 1) & 1, abort_flag);
        // All four warps take the same branch: they meet at named barrier 1 below.
        if (!bar_and(1, 128, got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + b * 128;
        f2 ss2 = f2_pack(0.f, 0.f);
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + cb * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float x0, x1;
            unpack2(pack_bf16x2(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), x0, x1);
            const f2 x2 = f2_pack(x0, x1);
            ss2 = f2_fma(x2, x2, ss2);
          }
        }
        float s0, s1;
        f2_unpack(ss2, s0, s1);
        const float ss = s0 + s1;
        const float nrm = sqrtf(ss);
        const float inv = round_bf16(__fdiv_rn(1.0f, sqrtf(nrm * nrm / 128.0f + p.eps)));
        const uint32_t ib = __float_as_uint(inv) >> 16, inv2 = ib | (ib << 16);
        uint8_t* gt = g_s + gs * RO_TILE;
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr + cb * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int col = cb * 32 + 8 * e4;  // 8 columns in one 16-byte chunk of a 64-column half
            uint4* cell = reinterpret_cast<uint4*>(gt + (col >> 6) * (RO_TILE / 2) + swz(erow, (col & 63) >> 3));
            const uint4 g4 = *cell;
            const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
            uint32_t yw[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int c = 8 * e4 + 2 * j;
              uint32_t rp = pack_bf16x2(__uint_as_float(v[c]), __uint_as_float(v[c + 1]));  // bf16(readout)
              rp = mul_bf16x2(rp, inv2);                                                     // bf16(. / rms)
              float a, b;
              unpack2(rp, a, b);
              const float2 wv = *reinterpret_cast<const float2*>(w_s + cb * 32 + c);
              f2_unpack(f2_mul(f2_pack(a, b), f2_pack(wv.x, wv.y)), a, b);
              yw[j] = mul_bf16x2(pack_bf16x2(a, b), gw[j]);                                  // bf16(bf16(. * w) * gate)
            }
            *cell = make_uint4(yw[0], yw[1], yw[2], yw[3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[b]);
        // The tile's rows are in shared memory: one thread stores it (rows past S are
        // clipped by the tensor map) once every epilogue thread's writes are visible
        // to the async proxy.
        fence_proxy_async_smem();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (issuer) {
          tma_store_4d(&tout, gt, 0, i * RO_TOK, h, f);
          tma_store_4d(&tout, gt + RO_TILE / 2, 64, i * RO_TOK, h, f);
          bulk_commit_group();
          bulk_wait_group_read<1>();  // the previous tile's store has read its buffer
          if (g > 0) mbar_arrive(&g_empty[(g - 1) % RO_GSTAGES]);
        }
      }
      if (!ok) break;
    }
    if (issuer) bulk_wait_group<0>();  // every store written before the CTA exits
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
                    int b_bf16, int* status, cudaStream_t stream) {
  using namespace vtc;
  CUtensorMap mk, mv;
  if (int rc = map_tokens(&mk, k, k_sf, k_ss, k_sh, F, S, H, ST_CH)) return rc;
  if (int rc = map_tokens(&mv, v, v_sf, v_ss, v_sh, F, S, H, ST_CH)) return rc;
  StatsParams p{static_cast<const uint16_t*>(beta), b_sf, b_ss, b_sh, A, B, b_bf16, S, H, F * H, status};
  int dev = 0, sms = 148;
  VDN_CUDA_TRY(cudaGetDevice(&dev));
  VDN_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = F * H < sms ? F * H : sms;
  static bool attr_set[2] = {false, false};
  if (features_applied) {
    if (!attr_set[0]) {
      VDN_CUDA_TRY(cudaFuncSetAttribute(stats_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ST_SMEM));
      attr_set[0] = true;
    }
    stats_tc_kernel<false><<<grid, ST_THREADS, ST_SMEM, stream>>>(mk, mv, p);
  } else {
    if (!attr_set[1]) {
      VDN_CUDA_TRY(cudaFuncSetAttribute(stats_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ST_SMEM));
      attr_set[1] = true;
    }
    stats_tc_kernel<true><<<grid, ST_THREADS, ST_SMEM, stream>>>(mk, mv, p);
  }
  VDN_LAUNCH_CHECK("vda statistics (tcgen05)");
  return VDN_OK;
}

bool tc_readout_supported(int d, const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh,
                          const void* state, const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh,
                          const void* out) {
  return d == 128 && vtc::strides_ok(q, q_sf, q_ss, q_sh) && vtc::is16(state) &&
         vtc::strides_ok(gate, g_sf, g_ss, g_sh) && vtc::is16(out);
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
  CUtensorMap mg, mo;
  if (int rc = map_tokens(&mg, gate, g_sf, g_ss, g_sh, F, S, H, RO_TOK)) return rc;
  // out: token-major [F, S, H, 128] bf16.
  const int64_t o_ss = (int64_t)H * 128;
  if (int rc = map_tokens(&mo, out, (int64_t)S * o_ss, o_ss, 128, F, S, H, RO_TOK)) return rc;
  ReadoutParams p{norm_w, eps, S, H, F * H, status};
  static bool attr_set = false;
  if (!attr_set) {
    VDN_CUDA_TRY(cudaFuncSetAttribute(readout_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)RO_SMEM));
    attr_set = true;
  }
  int dev = 0, sms = 148;
  VDN_CUDA_TRY(cudaGetDevice(&dev));
  VDN_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = F * H < sms ? F * H : sms;
  readout_tc_kernel<<<grid, RO_THREADS, RO_SMEM, stream>>>(mq, ms, mg, mo, p);
  VDN_LAUNCH_CHECK("vda readout (tcgen05)");
  return VDN_OK;
}

}  // namespace vdn
