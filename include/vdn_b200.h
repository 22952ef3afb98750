/* vdn_b200: B200-native (sm_100a) kernels for the VDN-H3 hybrid-attention DiT
 * block hot path, behind a plain C ABI.
 *
 * Every entry point takes raw device pointers, element counts and strides, and a
 * cudaStream_t (pass the caller's current stream; 0 is the legacy default
 * stream).  Nothing here allocates device memory: outputs and workspaces are
 * owned by the caller.  Every function returns VDN_OK (0) or an error code; the
 * message of the last error on the calling thread is vdn_last_error().  Bad
 * metadata is reported before any launch.  Launches are asynchronous; a device
 * fault surfaces at the caller's next synchronisation.
 *
 * Citations name the reference (ec-jt/vdn) interface each entry point replaces,
 * as path:line within that project.
 */
#ifndef VDN_B200_H
#define VDN_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VDN_ABI_VERSION 1

/* Status codes.  The Python layer maps VALUE -> ValueError, TYPE -> TypeError,
 * NONFINITE -> ValueError("nonfinite MXFP8 ..."), RUNTIME/TIMEOUT -> RuntimeError. */
#define VDN_OK 0
#define VDN_ERR_VALUE 1
#define VDN_ERR_TYPE 2
#define VDN_ERR_RUNTIME 3
#define VDN_ERR_NONFINITE 4
#define VDN_ERR_TIMEOUT 5

/* Element types for the dtype arguments. */
#define VDN_DTYPE_F32 0
#define VDN_DTYPE_BF16 1
#define VDN_DTYPE_F16 2

/* Activations of vdn_mxfp8_act_quantize. */
#define VDN_ACT_GELU_TANH 1
#define VDN_ACT_GELU_ERF 2
#define VDN_ACT_SWIGLU 3

/* Message of the last failing call on this thread ("" if none). */
const char* vdn_last_error(void);
int vdn_abi_version(void);
/* *supported = 1 when `device` is an sm_100 part this library was built for. */
int vdn_device_supported(int device, int* supported);

/* ------------------------------------------------------------------ MXFP8 */

/* Rows and K rounded up to multiples of 128.
 * Replaces padded_shape / scale_numel, src/models/ops/mxfp8_quant.py:15-23. */
int vdn_mxfp8_padded_shape(int64_t rows, int64_t k, int64_t* rows_padded, int64_t* k_padded);

/* bf16 [rows, k] (row_stride elements, K contiguous) -> E4M3 codes q [RP, KP]
 * (row-major, padding = exact zero) and E8M0 scales s [RP*KP/32] in the
 * SWIZZLE_32_4_4 layout.  Bit-exact with the reference rule.  When `nonfinite`
 * is not null, the count of 32-blocks holding a NaN/Inf input is ADDED to it.
 * Replaces quantize_activation / launch_quantize,
 * src/models/ops/mxfp8_quant.py:77-90, src/models/ops/mxfp8_kernels.py:30-58. */
int vdn_mxfp8_quantize(const void* x, int64_t rows, int64_t k, int64_t row_stride,
                       uint8_t* q, uint8_t* s, int* nonfinite, cudaStream_t stream);

/* vdn_mxfp8_quantize where logical column j of a row sits at element
 * (j / group) * group_stride + j % group of that row: quantises one half of
 * per-head interleaved [softmax | linear] rows (the Ulysses return buffer)
 * without a copy.  group a multiple of 32.  Same codes as vdn_mxfp8_quantize
 * on the gathered matrix. */
int vdn_mxfp8_quantize_grouped(const void* x, int64_t rows, int64_t k, int64_t row_stride,
                               int64_t group, int64_t group_stride, uint8_t* q, uint8_t* s,
                               int* nonfinite, cudaStream_t stream);

/* Fused activation producer: act(x) rounded to bf16, then quantised as above.
 * act = VDN_ACT_GELU_TANH / VDN_ACT_GELU_ERF read x [rows, k]; VDN_ACT_SWIGLU
 * reads x [rows, 2k] as (a | g) and produces a * silu(g).
 * Replaces launch_swiglu_quantize, src/models/ops/mxfp8_kernels.py:61-124,
 * 203-214 (the GELU forms are this build's analogue for a GELU FFN). */
int vdn_mxfp8_act_quantize(int act, const void* x, int64_t rows, int64_t k, int64_t row_stride,
                           uint8_t* q, uint8_t* s, int* nonfinite, cudaStream_t stream);

/* RMSNorm(x) * weight * (1 + scale[idx]) + shift[idx] -> bf16 (optionally
 * stored to y [rows, k] when y != NULL) -> MXFP8 codes/scales, plus a per-padded-
 * row finite byte finite[RP].  x, scale, shift bf16; weight fp32 or bf16;
 * indices int64 [rows].
 * Replaces launch_prenorm_quantize, src/models/ops/mxfp8_kernels.py:86-139, 217-229. */
int vdn_mxfp8_prenorm_quantize(const void* x, int64_t rows, int64_t k, int64_t x_stride,
                               const void* weight, int weight_dtype, float eps,
                               const void* scale, int64_t scale_stride, const void* shift,
                               int64_t shift_stride, const int64_t* indices, void* y,
                               uint8_t* q, uint8_t* s, uint8_t* finite, cudaStream_t stream);

/* One finite byte per 4096 elements: mode 0 float (dtype), 1 E4M3 codes
 * ((x & 127) != 127), 2 E8M0 bytes (x != 255).
 * Replaces finite_parts, src/models/ops/mxfp8_kernels.py:142-162. */
int vdn_finite_parts(const void* x, int64_t n, int dtype, int mode, uint8_t* parts,
                     cudaStream_t stream);

/* Host (CPU) weight quantiser, multithreaded; same outputs as the device
 * quantiser.  Returns VDN_ERR_NONFINITE on a NaN/Inf weight.
 * Replaces quantize_cpu, src/models/ops/mxfp8_quant.py:40-74. */
int vdn_mxfp8_quantize_host(const void* x, int dtype, int64_t rows, int64_t k,
                            int64_t row_stride, uint8_t* q, uint8_t* s, int num_threads);

/* Block-scaled MXFP8 GEMM on tcgen05 (kind::mxf8f6f4, scale_vec::1X):
 *   y[:rows_out, :n] = bf16(dequant(xq, xs) @ dequant(wq, ws)^T) (+ bias[n] bf16)
 * xq [m_pad, k_pad] / wq [n_pad, k_pad] E4M3 codes, xs / ws swizzled E8M0
 * scales, m_pad, n_pad, k_pad multiples of 128.  y bf16 with row stride ldy.
 * status: optional device int; set to VDN_ERR_TIMEOUT if a pipeline wait inside
 * the kernel gave up (the kernel then returns without finishing the tile).
 * Replaces MXFP8Linear.forward_quantized, src/models/ops/mxfp8_linear.py:60-93
 * (F.scaled_mm BlockWise1x32 / SWIZZLE_32_4_4). */
int vdn_mxfp8_gemm(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq, const uint8_t* ws,
                   const void* bias, int64_t m_pad, int64_t n, int64_t n_pad, int64_t k_pad,
                   int64_t rows_out, void* y, int64_t ldy, int* status, cudaStream_t stream);

/* vdn_mxfp8_gemm over two K ranges with one accumulator, and an optional gated
 * residual epilogue:
 *   r = bf16(dequant(x1) dequant(w1)^T + dequant(x2) dequant(w2)^T) (+ bias)
 *   y = resid != NULL ? bf16(resid + bf16(gate[col] * r)) : r
 * (k_pad2 = 0 for a single range).  y must not overlap resid (VDN_ERR_VALUE).  Covers the block's output projection
 * to_out(softmax) + to_out_linear(VDA) as one GEMM over K = 2 x 5120, and the
 * AdaLN gated residual adds, fused into the GEMM store.
 * Replaces HybridAttention's to_out + to_out_linear add (src/models/hybrid_attention.py:217-254)
 * and _post_ref (src/models/ops/fused_block.py:49-51) around MXFP8Linear. */
int vdn_mxfp8_gemm_fused(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq, const uint8_t* ws,
                         int64_t k_pad, const uint8_t* xq2, const uint8_t* xs2, const uint8_t* wq2,
                         const uint8_t* ws2, int64_t k_pad2, const void* bias, int64_t m_pad,
                         int64_t n, int64_t n_pad, int64_t rows_out, void* y, int64_t ldy,
                         const void* resid, int64_t ldr, const void* gate, int* status,
                         cudaStream_t stream);

/* vdn_mxfp8_gemm with a scatter epilogue: the 128 output columns of chunk c
 * (bf16, bias added) go to chunk_dst[c] + (dst_row0 + row) * dst_ld elements,
 * where chunk_dst is a DEVICE array of n / 128 bf16 pointers (local or peer
 * memory).  n % 128 == 0, dst_ld % 8 == 0, every pointer 16-byte aligned.  The
 * QKV projection uses it to store each head's q / k / v slice straight into
 * the receive buffer of the Ulysses rank that owns the head.
 * Replaces MXFP8Linear (src/models/ops/mxfp8_linear.py:60-102) followed by the
 * sequence -> heads all-to-all (src/inference/utils/ulysses_runtime.py:451-519). */
int vdn_mxfp8_gemm_scatter(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq, const uint8_t* ws,
                           int64_t k_pad, const void* bias, int64_t m_pad, int64_t n, int64_t n_pad,
                           int64_t rows_out, const uint64_t* chunk_dst, int64_t dst_ld,
                           int64_t dst_row0, int* status, cudaStream_t stream);

/* vdn_mxfp8_gemm whose epilogue applies an activation and quantises: with
 * r = bf16(bf16(dequant(x) dequant(w)^T) + bias), the bf16 value act(r)
 * (act = VDN_ACT_GELU_TANH or 0 for none) is stored as
 * MXFP8: codes q [m_pad, n] and swizzled scales s [m_pad * n / 32], rows in
 * [rows_out, m_pad) zero.  n % 128 == 0; q, bias 16-byte aligned.  Bit-identical
 * to vdn_mxfp8_gemm followed by vdn_mxfp8_act_quantize, without the bf16
 * round trip through HBM: the FFN up projection feeding the down projection.
 * Replaces MXFP8Linear + the GELU/SwiGLU producer of src/models/ops/fused_block.py:82-105
 * and src/models/ops/mxfp8_kernels.py:61-124. */
int vdn_mxfp8_gemm_act_quantize(const uint8_t* xq, const uint8_t* xs, const uint8_t* wq,
                                const uint8_t* ws, int64_t k_pad, const void* bias, int64_t m_pad,
                                int64_t n, int64_t n_pad, int64_t rows_out, int act, uint8_t* q,
                                uint8_t* s, int* status, cudaStream_t stream);

/* bf16 GEMM with the gate epilogue: y[:rows, :n] = act(bf16(x w^T + bias)) with fp32
 * accumulation and the bias added before the single bf16 rounding (an eager bf16
 * nn.Linear), act = sigmoid followed by bf16 rounding on columns < n_sig (torch.sigmoid
 * on the bf16 tensor), identity after.  x [rows, k] (row stride ldx), w [n, k] (row
 * stride ldw), y [rows, n] (row stride ldy): bf16, 16-byte aligned, strides multiples
 * of 8 elements; k % 64 == 0; bias [n] bf16 or NULL.  tcgen05 kind::f16, TMA in and out.
 * Replaces the gate projections of src/models/hybrid_attention.py:108-255 (softmax gate
 * and beta projection, sigmoid) and OutputGate of src/models/attention_gates.py:13-55
 * (down, then up + sigmoid): the block calls it once for [softmax gate | beta | output
 * gate down] over y1 and once for the output gate's up projection. */
int vdn_gate_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias, int64_t rows,
                  int64_t n, int64_t k, int64_t n_sig, void* y, int64_t ldy, int* status, cudaStream_t stream);

/* Window-softmax combine: merges n_partials dense attentions of query frame f
 * against key frame f + delta_j (outs[j] bf16 [rows_j, H*d] token-major, lses[j]
 * fp32 [batches_j, H, S]; batch = f - batch0[j], valid for frame_lo[j] <= f <=
 * frame_hi[j]) by their log-sum-exps, rounds to bf16, multiplies by the softmax
 * gate (bf16, element (t, h) at t*g_ss + h*g_sh) and writes bf16 out (element
 * (t, h, j) at t*out_ld + h*out_hs + j) and/or MXFP8 codes q [RP, H*d] and
 * swizzled scales s.
 * Replaces the window softmax combine and apply_softmax_gate of
 * src/models/softmax_attention/decomposed.py and src/models/hybrid_attention.py:165-222. */
int vdn_window_merge(int n_partials, const void* const* outs, const float* const* lses,
                     const int* batch0, const int* frame_lo, const int* frame_hi, int F, int S,
                     int H, int d, const void* gate, int64_t g_ss, int64_t g_sh, void* out_bf16,
                     int64_t out_ld, int64_t out_hs, uint8_t* q, uint8_t* s, cudaStream_t stream);

/* ---------------------------------------------------------- peer memory */

#define VDN_IPC_HANDLE_BYTES 64

/* Zero-filled device buffer for exchange through CUDA IPC (cudaMalloc'd, so it
 * is the base of its allocation), and its release. */
int vdn_peer_alloc(size_t bytes, void** ptr);
int vdn_peer_free(void* ptr);

/* CUDA IPC: export a vdn_peer_alloc buffer as VDN_IPC_HANDLE_BYTES bytes, map a
 * peer's exported buffer into this process (peer access enabled), unmap it. */
int vdn_ipc_handle(const void* ptr, void* handle);
int vdn_ipc_open(const void* handle, void** ptr);
int vdn_ipc_close(void* ptr);

/* Stream-ordered device copy (local or peer memory; a copy engine, no SM). */
int vdn_copy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream);

/* Copies `bytes` (a multiple of 16, 16-byte aligned) from src to each of the
 * ndst <= 8 destinations (host array of device pointers, local or peer) in one
 * launch: the all-gather of small per-token side inputs. */
int vdn_peer_broadcast(const void* src, size_t bytes, int ndst, void* const* dsts, cudaStream_t stream);

/* Cross-GPU rendezvous on the stream: the epoch is *counter + 1 (counter: this
 * rank's uint64 on the device, zero-initialised, advanced by each call, so the
 * launch can be replayed from a CUDA graph).  Publishes the epoch into slot
 * `rank` of every rank's uint64 flag array (flag_arrays[p], host array of device
 * pointers, p < nranks <= 8; a system-scope release after all earlier work of
 * the stream) and waits until all nranks slots of this rank's array (my_flags)
 * hold at least the epoch.  Later work on the stream then sees every rank's
 * stores made before its matching call.  Every rank makes the same sequence of
 * calls.  Each wait gives up after 2 s and sets *status (optional device int) to
 * VDN_ERR_TIMEOUT. */
int vdn_peer_fence(int nranks, void* const* flag_arrays, const void* my_flags, int rank,
                   uint64_t* counter, int* status, cudaStream_t stream);

/* Heads -> sequence return of a head-sharded bf16 output as MXFP8: element
 * (t, j, e) of src (t < rows, j < heads_local, e < d) sits at t*row_stride +
 * j*head_stride + e.  Each 32-element block is quantised with the MXFP8 rule
 * and stored, with its E8M0 byte, into the operand of the rank that owns token
 * t (row_starts[p] <= t < row_starts[p + 1], host array of nranks + 1): codes
 * [rp_p, kp] at dst_codes[p], swizzled scales at dst_scales[p] (host arrays of
 * device pointers, local or peer), column (head0 + j) * d + e.  nranks <= 8.
 * Replaces the heads -> sequence all-to-all (src/inference/utils/ulysses_runtime.py:522-582)
 * and the MXFP8 quantisation of to_out / to_out_linear inputs
 * (src/models/ops/mxfp8_quant.py:77-90). */
int vdn_mxfp8_quantize_scatter(const void* src, int64_t rows, int heads_local, int d,
                               int64_t row_stride, int64_t head_stride, int head0, int64_t kp,
                               int nranks, const int64_t* row_starts, void* const* dst_codes,
                               void* const* dst_scales, int* nonfinite, cudaStream_t stream);

/* -------------------------------------------------------------------- VDA */

/* Separable short conv of one projection (depthwise 5x5 spatial per frame, then
 * depthwise 5-tap temporal across frames, zero padding, no bias): x [F*gh*gw, C]
 * bf16 rows (stride x_ld, frame-major, (y, x) row-major in a frame) ->
 * out [F*gh*gw, C] bf16 (stride out_ld).  w_spatial [25, C] and w_temporal [5, C]
 * bf16, tap-major; scratch holds F*gh*gw*C bf16 (the spatial half).  C % 8 == 0,
 * pointers 16-byte aligned, strides % 8 == 0.  The spatial half is rounded to
 * bf16; the temporal half sums its five exact products in fp32 (taps in order)
 * and rounds once.
 * Replaces LinearAttentionSepConv.spatial + _temporal_conv,
 * src/models/linear_attention/features.py:133-209 and :12-40. */
int vdn_sepconv(const void* x, int64_t x_ld, int F, int gh, int gw, int C, const void* w_spatial,
                const void* w_temporal, void* scratch, void* out, int64_t out_ld, cudaStream_t stream);

/* Per-frame column sums of bf16 rows: out [frames, width] fp32, out[f, c] = (sum of
 * x[r, c] over r in [bounds[f], bounds[f + 1])) / divisor, in a fixed summation order
 * (the same result on every run).  x [rows, width] bf16 with row stride ld (elements;
 * width and ld multiples of 8, x 16-byte aligned); bounds host int32 [frames + 1],
 * nondecreasing within [0, rows] (an empty range gives zeros); frames <= 1024.
 * divisor = tokens per frame gives the frame mean, 1 the sums of a sequence shard.
 * Replaces the frame mean of BidirectionalLinearBranch, src/models/linear_attention/
 * branch.py:450-452, and UlyssesRuntime._local_video_frame_sums,
 * src/inference/utils/ulysses_runtime.py:606-635. */
int vdn_frame_sums(const void* x, int64_t ld, int64_t rows, int64_t width, const int32_t* bounds, int frames,
                   float divisor, float* out, cudaStream_t stream);

/* FrameKDAAlpha: alpha [F, heads, d] fp32 = exp(-exp(a_log[h]) * softplus(
 * (frame_mean @ down_w^T) @ up_w^T + dt_bias)), softplus threshold 20.
 * frame_mean [F, hidden], down_w [r, hidden], up_w [heads*d, r], dt_bias
 * [heads*d], a_log [heads] (fp32, contiguous; pass the selected heads' rows for
 * a head shard); scratch holds F*r floats.
 * Replaces FrameKDAAlpha.forward, src/models/linear_attention/layers.py:36-69. */
int vdn_frame_alpha(const float* frame_mean, int F, int hidden, const float* down_w, int r,
                    const float* up_w, const float* dt_bias, const float* a_log, int heads, int d,
                    float* scratch, float* out, cudaStream_t stream);


/* Per (frame, head) delta-rule factors, d in {64, 128}, n matrices:
 *   T = diag(alpha) (I + A)^-1,  J = B (I + A)^-1    (alpha NULL = ones)
 * A, B, T, J fp32 [n, d, d]; alpha fp32 [n, d].  I + A must be SPD.
 * Replaces paper_delta_factors, src/models/linear_attention/paper_factor.py:133-186,
 * and VdnDelta.factor_apply, src/models/linear_attention/delta_rule.py:45-60. */
int vdn_delta_factors(const float* A, const float* B, const float* alpha, int64_t n, int d,
                      float* T, float* J, cudaStream_t stream);

/* Frame statistics from RAW projections (SiLU + L2 over d for k, SiLU for v,
 * rounded to bf16 as the feature path does, then multiplied by beta):
 *   A[f,h] = sym(sum_s (k beta)(k)^T) fp32,  B[f,h] = bf16(sum_s bf16(v beta) k^T)
 * Element (f, s, h, :) of k / v / beta lives at f*stride_f + s*stride_s + h*stride_h
 * (elements; d contiguous for k and v).  A, B fp32 [F, H, d, d].
 * Replaces frame_statistics, src/models/linear_attention/scan.py:113-267, and
 * paper_statistics, src/models/linear_attention/paper_stack.py:51-110. */
int vdn_vda_statistics(const void* k, int64_t k_sf, int64_t k_ss, int64_t k_sh,
                       const void* v, int64_t v_sf, int64_t v_ss, int64_t v_sh,
                       const void* beta, int64_t b_sf, int64_t b_ss, int64_t b_sh,
                       int features_applied, int F, int S, int H, int d,
                       float* A, float* B, cudaStream_t stream);

/* Forward and reverse scans s_t = s_{t-1} T_t + J_t over F frames, started from
 * seed [H, d, d] (NULL = zero).  prefix / suffix fp32 [F, H, d, d].
 * Replaces _run_scans / _run_scans_inference, src/models/linear_attention/scan.py:270-355. */
int vdn_vda_scan(const float* T, const float* J, const float* seed, int F, int H, int d,
                 float* prefix, float* suffix, cudaStream_t stream);

/* State outside each frame's inclusive window [lo, hi] (bounds: host int32
 * [F][2], F <= 1024), decayed into the frame by prod(alpha) when bridge != 0:
 *   out[t] = prefix[lo-1] * prod_{lo..t} alpha + suffix[hi+1] * prod_{t..hi} alpha
 * with the seed (or zero) past the clip ends.  out [F, H, d, d], out_dtype
 * VDN_DTYPE_F32 or VDN_DTYPE_BF16.
 * Replaces gather_linear_state, src/models/linear_attention/scan.py:361-496, and
 * paper_gather, src/models/linear_attention/paper_stack.py:239-263. */
int vdn_vda_gather(const float* prefix, const float* suffix, const float* alpha,
                   const int32_t* bounds, const float* seed, int bridge, int F, int H, int d,
                   void* out, int out_dtype, cudaStream_t stream);

/* Readout and epilogue: q features (SiLU + L2, bf16) times state^T (bf16
 * [F, H, d, d]), RMSNorm over d (eps) times norm_weight (fp32 [d]) times gate,
 * stored token-major out [F*S, H*d] bf16.  q and gate addressing as in
 * vdn_vda_statistics.
 * Replaces the readout + linear_epilogue of branch.py:470-482 / 560-563 and
 * vdn_linear_epilogue, src/models/linear_attention/paper_sglang.py:377-437. */
int vdn_vda_readout(const void* q, int64_t q_sf, int64_t q_ss, int64_t q_sh,
                    const void* state, const void* gate, int64_t g_sf, int64_t g_ss, int64_t g_sh,
                    const float* norm_weight, float eps, int F, int S, int H, int d,
                    void* out, cudaStream_t stream);

/* The two tensor-core stages vdn_vda_forward runs for d = 128 in place of
 * vdn_delta_factors + vdn_vda_scan (no separate counterpart in the reference: together
 * they compute delta_rule.py:45-60 and scan.py:176-261 with the injection J = B inv
 * folded into each scan step).
 * vdn_vda_factor_inverse: inv = (I + A)^-1 for n fp32 [128, 128] matrices A, written
 * as three bf16 planes whose sum is the fp32 inverse, each plane in the 128B-swizzled
 * K-major tcgen05 operand layout: 98304 bytes per matrix at `planes` (16-byte aligned).
 * vdn_vda_scan_tc: P_f = (P_{f-1} diag(alpha_f) + B_f) inv_f over the F frames in both
 * directions (forward into prefix, reverse into suffix, [F, H, 128, 128] fp32), from
 * the planes of [F, H] inverses, B [F, H, 128, 128] fp32, alpha [F, H, 128] fp32 and an
 * optional seed [H, 128, 128]; status (optional int32) receives VDN_ERR_TIMEOUT if a
 * bounded wait gave up.  Operands 16-byte aligned; prefix and suffix 32-byte aligned
 * (the banks leave in 32-byte stores). */
int vdn_vda_factor_inverse(const float* A, int64_t n, void* planes, cudaStream_t stream);
int vdn_vda_scan_tc(const void* planes, const float* B, const float* alpha, const float* seed, int F, int H,
                    float* prefix, float* suffix, int* status, cudaStream_t stream);
/* vdn_vda_scan_tc with B in bf16 [F, H, 128, 128] (the values the statistics produce are
 * bf16 already): B_f reaches the kernel by TMA instead of per-thread loads.  The form
 * vdn_vda_forward uses for d = 128. */
int vdn_vda_scan_tc_bf16(const void* planes, const void* B, const float* alpha, const float* seed, int F,
                         int H, float* prefix, float* suffix, int* status, cudaStream_t stream);

/* Workspace bytes vdn_vda_forward needs for this geometry. */
size_t vdn_vda_workspace_size(int F, int S, int H, int d);

/* The whole VDA branch body over the frames it owns: statistics, factors,
 * bidirectional scans, boundary gather, readout, RMSNorm and gate.
 * q, k, v [F*S, H, d] bf16 with token stride qkv_ss and head stride qkv_sh
 * (shared by the three), beta [F*S, H] bf16 (b_ss, b_sh), gate [F*S, H, d] bf16
 * (g_ss, g_sh), alpha fp32 [F, H, d] contiguous, norm_weight fp32 [d], bounds
 * host int32 [F][2], seed fp32 [H, d, d] or NULL, out bf16 [F*S, H*d]; workspace
 * (vdn_vda_workspace_size bytes) 32-byte aligned.
 * Replaces BidirectionalLinearBranch._readout / _readout_inference / paper_readout,
 * src/models/linear_attention/branch.py:404-563, paper_stack.py:266-318. */
int vdn_vda_forward(const void* q, const void* k, const void* v, int64_t qkv_ss, int64_t qkv_sh,
                    const void* beta, int64_t b_ss, int64_t b_sh,
                    const void* gate, int64_t g_ss, int64_t g_sh,
                    const float* alpha, const float* norm_weight, float eps,
                    const int32_t* bounds, const float* seed, int bridge,
                    int F, int S, int H, int d, void* out,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* vdn_vda_forward without a workspace argument, for callers that cannot give
 * this library device memory or let it call cudaMalloc (a host engine that owns
 * all device memory through its own pool, or a latency-critical loop that cannot
 * take cudaMalloc's device synchronisation).  Same kernels and results as
 * vdn_vda_forward; the scratch is a 64 MiB array built into the library.
 * Geometries whose vdn_vda_workspace_size exceeds 64 MiB return VDN_ERR_VALUE
 * (at d = 128: 20 frames x 10 heads fit, 21 x 10 do not).  The first call on a
 * device looks the array's address up; under CUDA's lazy module loading that is
 * also when the device reserves the 64 MiB (kept until the process exits) and
 * it may synchronise the device, so make one warm-up call outside latency-
 * critical code and before any stream capture.  The address is looked up again
 * if the device's context was recreated.  All calls share the array, so calls
 * that overlap on the GPU race.  It allocates nothing.  This entry point has no
 * counterpart in the reference (ec-jt/vdn): its branch body always allocates
 * through PyTorch. */
int vdn_vda_forward_noalloc(const void* q, const void* k, const void* v, int64_t qkv_ss,
                            int64_t qkv_sh, const void* beta, int64_t b_ss, int64_t b_sh,
                            const void* gate, int64_t g_ss, int64_t g_sh,
                            const float* alpha, const float* norm_weight, float eps,
                            const int32_t* bounds, const float* seed, int bridge,
                            int F, int S, int H, int d, void* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VDN_B200_H */
