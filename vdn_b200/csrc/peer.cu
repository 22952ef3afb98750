// Peer memory for the Ulysses exchange: device buffers shared between the
// ranks of one node through CUDA IPC, and the kernel that returns head-sharded
// attention outputs to their sequence owners as MXFP8.
//
// The reference moves activations with NCCL all-to-all
// (src/inference/utils/ulysses_runtime.py:451-582): sequence -> heads before
// attention and heads -> sequence after it.  Here the producers write straight
// into the consumer's memory over NVLink instead: the QKV GEMM epilogue stores
// each head's q / k / v slice into the receive buffer of the rank that owns
// the head (vdn_mxfp8_gemm_scatter), and vdn_mxfp8_quantize_scatter quantises
// each (token, head) slice of the attention outputs and stores the E4M3 codes
// and E8M0 scale bytes into the owner rank's padded GEMM operand.  Plain peer
// loads and stores only: no multicast objects.
#include "common.cuh"
#include "mxfp8.cuh"

namespace vdn {

constexpr int kMaxRanks = 8;

struct Route {
  int nranks;
  int64_t start[kMaxRanks + 1];  // row_starts: rank p owns global rows [start[p], start[p+1])
  uint8_t* codes[kMaxRanks];     // rank p's codes [rp_p, kp]
  uint8_t* scales[kMaxRanks];    // rank p's swizzled scales
};

// One thread per 32-element block of a (token, head) slice.  WORD: d % 128 == 0,
// so the four blocks of a 128-column group sit in four adjacent lanes and their
// scale bytes leave as one 32-bit word (the SWIZZLE_32_4_4 layout keeps c..c+3
// of a row contiguous).
template <bool VEC, bool WORD>
__global__ void __launch_bounds__(256) quantize_scatter_kernel(
    const uint16_t* __restrict__ src, int64_t rows, int hl, int d, int64_t rs, int64_t hs, int head0,
    int64_t kp, const Route route, int* __restrict__ nonfinite) {
  const int bph = d >> 5;
  const int64_t per_row = (int64_t)hl * bph;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = g < rows * per_row;
  int64_t t = 0;
  int j = 0, b = 0;
  if (active) {
    t = g / per_row;
    const int64_t rem = g - t * per_row;
    j = (int)(rem / bph);
    b = (int)(rem - (int64_t)j * bph);
  }
  float v[32];
  bool bad = false;
  if (active) {
    const uint16_t* x = src + t * rs + (int64_t)j * hs + 32 * b;
    if (VEC) {
#pragma unroll
      for (int i = 0; i < 4; ++i) unpack8(__ldg(reinterpret_cast<const uint4*>(x) + i), v + 8 * i);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = bf16_bits_to_f32(x[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
  uint32_t amax_bits = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    bad |= !isfinite(v[i]);
    const uint32_t bits = __float_as_uint(v[i]) & 0x7FFFFFFFu;
    amax_bits = bits > amax_bits ? bits : amax_bits;
  }
  float inv;
  const uint32_t sbyte = e8m0_from_amax_bits(amax_bits, &inv);
  uint32_t word = 0;
  if (WORD) {
    const unsigned lane = threadIdx.x & 31;
    word = sbyte << (8 * (lane & 3));
    word |= __shfl_xor_sync(0xffffffffu, word, 1);
    word |= __shfl_xor_sync(0xffffffffu, word, 2);
  }
  if (!active) return;
  int p = 0;
  while (p + 1 < route.nranks && t >= route.start[p + 1]) ++p;
  const int64_t r = t - route.start[p];
  const int64_t c = (int64_t)(head0 + j) * bph + b;
  uint32_t packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    packed[i] = e4m3x4(v[4 * i] * inv, v[4 * i + 1] * inv, v[4 * i + 2] * inv, v[4 * i + 3] * inv);
  uint4* qp = reinterpret_cast<uint4*>(route.codes[p] + r * kp + c * 32);
  qp[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  qp[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  if (WORD) {
    if ((b & 3) == 0) *reinterpret_cast<uint32_t*>(route.scales[p] + scale_offset(r, c, kp)) = word;
  } else {
    route.scales[p][scale_offset(r, c, kp)] = (uint8_t)sbyte;
  }
  if (bad && nonfinite) atomicAdd(nonfinite, 1);
}

struct PeerSet {
  int n;
  uint8_t* ptr[kMaxRanks];
};

// Copies `bytes` (a multiple of 16) from src to every destination: each thread
// loads one 16-byte vector and stores it to all of them.
__global__ void __launch_bounds__(256) broadcast_kernel(const uint4* __restrict__ src, int64_t n16,
                                                        const PeerSet dst) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = __ldg(src + i);
#pragma unroll 1
    for (int p = 0; p < dst.n; ++p) reinterpret_cast<uint4*>(dst.ptr[p])[i] = v;
  }
}

// Cross-GPU rendezvous: the epoch is this rank's counter + 1 (a device word, so
// the same launch can be replayed from a CUDA graph).  Thread p publishes it into
// slot `rank` of rank p's flag array (a system-scope release, ordered after every
// earlier kernel of this stream), then waits (acquire, bounded by kFenceLimitNs)
// until every rank has published it into this rank's array; thread 0 then
// stores the new epoch into the counter.  A timeout sets *status.
constexpr uint64_t kFenceLimitNs = 2000000000ull;

__global__ void peer_fence_kernel(const PeerSet flags, const uint64_t* my_flags, int rank,
                                  uint64_t* counter, int* status) {
  const int p = threadIdx.x;
  const uint64_t epoch = *counter + 1;
  if (p < flags.n) {
    uint64_t* slot = reinterpret_cast<uint64_t*>(flags.ptr[p]) + rank;
    asm volatile("fence.sc.sys;\n\tst.release.sys.global.u64 [%0], %1;" ::"l"(slot), "l"(epoch) : "memory");
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    while (true) {
      uint64_t v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(my_flags + p) : "memory");
      if (v >= epoch) break;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > kFenceLimitNs) {
        if (status) atomicExch(status, VDN_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
  if (p == 0) *counter = epoch;
}

}  // namespace vdn

using namespace vdn;

extern "C" {

int vdn_peer_alloc(size_t bytes, void** ptr) {
  VDN_CHECK_ARG(ptr && bytes > 0, "need a positive size and an output pointer");
  *ptr = nullptr;
  VDN_CUDA_TRY(cudaMalloc(ptr, bytes));
  const cudaError_t err = cudaMemset(*ptr, 0, bytes);
  if (err != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return set_error(VDN_ERR_RUNTIME, "cudaMemset: %s", cudaGetErrorString(err));
  }
  return VDN_OK;
}

int vdn_peer_free(void* ptr) {
  if (!ptr) return VDN_OK;
  VDN_CUDA_TRY(cudaFree(ptr));
  return VDN_OK;
}

int vdn_ipc_handle(const void* ptr, void* handle) {
  VDN_CHECK_ARG(ptr && handle, "null pointer");
  cudaIpcMemHandle_t h;
  VDN_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  memcpy(handle, &h, sizeof(h));
  return VDN_OK;
}

int vdn_ipc_open(const void* handle, void** ptr) {
  VDN_CHECK_ARG(ptr && handle, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  VDN_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return VDN_OK;
}

int vdn_ipc_close(void* ptr) {
  if (!ptr) return VDN_OK;
  VDN_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return VDN_OK;
}

int vdn_copy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  if (bytes == 0) return VDN_OK;
  VDN_CHECK_ARG(dst && src, "null pointer");
  VDN_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, stream));
  return VDN_OK;
}

int vdn_peer_broadcast(const void* src, size_t bytes, int ndst, void* const* dsts, cudaStream_t stream) {
  VDN_CHECK_ARG(ndst >= 0 && ndst <= kMaxRanks, "at most %d destinations", kMaxRanks);
  if (bytes == 0 || ndst == 0) return VDN_OK;
  VDN_CHECK_ARG(src && dsts && aligned16(src) && bytes % 16 == 0,
                "source must be 16-byte aligned with a size that is a multiple of 16");
  PeerSet set;
  set.n = ndst;
  for (int p = 0; p < kMaxRanks; ++p) set.ptr[p] = nullptr;
  for (int p = 0; p < ndst; ++p) {
    VDN_CHECK_ARG(dsts[p] && aligned16(dsts[p]), "destinations must be non-null and 16-byte aligned");
    set.ptr[p] = static_cast<uint8_t*>(dsts[p]);
  }
  const int64_t n16 = (int64_t)(bytes / 16);
  const int64_t want = (n16 + 255) / 256;
  const unsigned grid = (unsigned)(want < 1184 ? want : 1184);
  broadcast_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(src), n16, set);
  VDN_LAUNCH_CHECK("peer broadcast");
  return VDN_OK;
}

int vdn_peer_fence(int nranks, void* const* flag_arrays, const void* my_flags, int rank,
                   uint64_t* counter, int* status, cudaStream_t stream) {
  VDN_CHECK_ARG(nranks >= 1 && nranks <= kMaxRanks, "nranks must lie in [1, %d]", kMaxRanks);
  VDN_CHECK_ARG(rank >= 0 && rank < nranks && flag_arrays && my_flags && counter, "bad fence arguments");
  VDN_CHECK_ARG((reinterpret_cast<uintptr_t>(counter) & 7) == 0, "counter must be 8-byte aligned");
  PeerSet set;
  set.n = nranks;
  for (int p = 0; p < kMaxRanks; ++p) set.ptr[p] = nullptr;
  for (int p = 0; p < nranks; ++p) {
    VDN_CHECK_ARG(flag_arrays[p] && (reinterpret_cast<uintptr_t>(flag_arrays[p]) & 7) == 0,
                  "flag arrays must be non-null and 8-byte aligned");
    set.ptr[p] = static_cast<uint8_t*>(flag_arrays[p]);
  }
  peer_fence_kernel<<<1, 32, 0, stream>>>(set, static_cast<const uint64_t*>(my_flags), rank, counter, status);
  VDN_LAUNCH_CHECK("peer fence");
  return VDN_OK;
}

int vdn_mxfp8_quantize_scatter(const void* src, int64_t rows, int heads_local, int d,
                               int64_t row_stride, int64_t head_stride, int head0, int64_t kp,
                               int nranks, const int64_t* row_starts, void* const* dst_codes,
                               void* const* dst_scales, int* nonfinite, cudaStream_t stream) {
  VDN_CHECK_ARG(rows >= 0 && heads_local > 0 && d > 0 && d % 32 == 0, "bad extents");
  VDN_CHECK_ARG(nranks >= 1 && nranks <= kMaxRanks, "nranks must lie in [1, %d]", kMaxRanks);
  VDN_CHECK_ARG(row_starts && dst_codes && dst_scales, "null route arrays");
  VDN_CHECK_ARG(kp % 128 == 0 && head0 >= 0 && (int64_t)(head0 + heads_local) * d <= kp,
                "kp must be a multiple of 128 holding columns [head0 * d, (head0 + heads_local) * d)");
  VDN_CHECK_ARG(row_starts[0] == 0 && row_starts[nranks] == rows, "row_starts must span [0, rows]");
  Route route;
  route.nranks = nranks;
  for (int p = 0; p <= kMaxRanks; ++p) route.start[p] = p <= nranks ? row_starts[p] : rows;
  for (int p = 0; p < kMaxRanks; ++p) {
    route.codes[p] = nullptr;
    route.scales[p] = nullptr;
  }
  for (int p = 0; p < nranks; ++p) {
    VDN_CHECK_ARG(row_starts[p + 1] >= row_starts[p], "row_starts must be nondecreasing");
    VDN_CHECK_ARG(dst_codes[p] && dst_scales[p] && aligned16(dst_codes[p]),
                  "destination of rank %d must be non-null with 16-byte aligned codes", p);
    route.codes[p] = static_cast<uint8_t*>(dst_codes[p]);
    route.scales[p] = static_cast<uint8_t*>(dst_scales[p]);
  }
  if (rows == 0) return VDN_OK;
  VDN_CHECK_ARG(src, "null source");
  const bool vec = aligned16(src) && row_stride % 8 == 0 && head_stride % 8 == 0;
  const bool word = d % 128 == 0;
  const int64_t threads = rows * heads_local * (d / 32);
  const unsigned grid = (unsigned)((threads + 255) / 256);
  const uint16_t* s = static_cast<const uint16_t*>(src);
#define VDN_SCATTER(V, W)                                                                   \
  quantize_scatter_kernel<V, W><<<grid, 256, 0, stream>>>(s, rows, heads_local, d, row_stride, \
                                                          head_stride, head0, kp, route, nonfinite)
  if (vec && word) VDN_SCATTER(true, true);
  else if (vec) VDN_SCATTER(true, false);
  else if (word) VDN_SCATTER(false, true);
  else VDN_SCATTER(false, false);
#undef VDN_SCATTER
  VDN_LAUNCH_CHECK("mxfp8 quantize scatter");
  return VDN_OK;
}

}  // extern "C"
