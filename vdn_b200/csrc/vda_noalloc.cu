// vdn_vda_forward_noalloc: the VDA branch body for callers that cannot allocate
// device memory.
//
// Some hosts of this library cannot hand it a workspace and cannot let it call
// cudaMalloc: an engine that owns every byte of device memory through its own
// pool and forbids allocations from plugins, or a latency-critical loop where
// cudaMalloc's implicit device synchronisation is not acceptable.  This entry
// point runs exactly the same kernels as vdn_vda_forward, but its scratch
// memory (statistics / factors, both scan banks and the gathered state) lives
// in one file-scope device array compiled into the library.
//
// Limits and rules:
//  * The array holds kScratchBytes = 64 MiB.  A geometry whose
//    vdn_vda_workspace_size exceeds it is rejected with VDN_ERR_VALUE before
//    anything is launched; at d = 128 and 10 heads that is 21 frames or more
//    (20 frames x 10 heads needs 65,536,000 bytes and is accepted).
//  * Host code cannot use the array's name as a device address.  The first call
//    on each device (with that device current) looks the address up with
//    cudaGetSymbolAddress.  With CUDA's lazy module loading that first lookup is
//    also when the driver loads this file's module and reserves the 64 MiB on
//    the device, which can synchronise the device: make one warm-up call outside
//    any latency-critical loop and before any stream capture.  From then on the
//    device keeps the 64 MiB until the process exits.
//  * The address is cached per device together with the identity of the CUDA
//    context it was looked up in; if the device was reset and the context
//    recreated, the next call looks the address up again instead of using a
//    stale one.
//  * Every call shares the one array and it keeps the previous call's contents.
//    Nothing in it needs to start at zero (every region is written before it is
//    read), but calls whose work overlaps on the GPU (other streams, other host
//    threads) race on it: serialise them.
#include "common.cuh"

#include <cuda.h>

#include <mutex>

namespace vdn {
namespace {

constexpr size_t kScratchBytes = 64ull << 20;

static __device__ __align__(256) unsigned char g_vda_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(fn);
}

// Unique id of the calling thread's current CUDA context (0 when unknown).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of g_vda_scratch on the current device, looked up once per
// device and context.
int scratch_address(void** out) {
  int dev = 0;
  VDN_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(VDN_ERR_RUNTIME, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_scratch_ptr[dev] || ctx == 0 || ctx != g_scratch_ctx[dev]) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_vda_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return set_error(VDN_ERR_RUNTIME, "cudaGetSymbolAddress(VDA scratch) failed: %s",
                       cudaGetErrorString(err));
    g_scratch_ptr[dev] = ptr;
    // The lookup made the context current if it was not yet; record it now.
    g_scratch_ctx[dev] = current_context_id();
  }
  *out = g_scratch_ptr[dev];
  return VDN_OK;
}

}  // namespace
}  // namespace vdn

extern "C" int vdn_vda_forward_noalloc(const void* q, const void* k, const void* v, int64_t qkv_ss,
                                       int64_t qkv_sh, const void* beta, int64_t b_ss, int64_t b_sh,
                                       const void* gate, int64_t g_ss, int64_t g_sh,
                                       const float* alpha, const float* norm_weight, float eps,
                                       const int32_t* bounds, const float* seed, int bridge, int F,
                                       int S, int H, int d, void* out, cudaStream_t stream) {
  if (F < 1 || S < 1 || H < 1 || (d != 64 && d != 128))
    return vdn::set_error(VDN_ERR_VALUE, "bad VDA geometry F=%d S=%d H=%d d=%d", F, S, H, d);
  const size_t need = vdn_vda_workspace_size(F, S, H, d);
  if (need > vdn::kScratchBytes)
    return vdn::set_error(VDN_ERR_VALUE,
                          "geometry needs %zu scratch bytes; the built-in scratch holds %zu "
                          "(use vdn_vda_forward with a caller workspace)",
                          need, vdn::kScratchBytes);
  void* scratch = nullptr;
  if (int rc = vdn::scratch_address(&scratch)) return rc;
  return vdn_vda_forward(q, k, v, qkv_ss, qkv_sh, beta, b_ss, b_sh, gate, g_ss, g_sh, alpha,
                         norm_weight, eps, bounds, seed, bridge, F, S, H, d, out, scratch,
                         vdn::kScratchBytes, stream);
}
