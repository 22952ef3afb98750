// Test infrastructure, not product code: a C-ABI launcher for the reference's own
// sm_100 delta-rule factor kernel, so the GPU tests can check the product's factor
// stage against it and time the two side by side.  Only tests/ load the library.
//
// The kernel itself is not in this repository.  oracle/build_ref.py compiles this
// file with -I pointing at the reference's src/models/ops/csrc, where
// vdn_delta_factors.cuh (vdn_delta_factors_kernel, :200-306) lies, using the flags of
// the reference's own builder (src/models/linear_attention/paper_factor.py:85-93:
// -O3 -std=c++17, compute_XY/sm_XY of the device).  The launch shape is the one its
// host wrapper uses (src/models/ops/csrc/vdn_delta_factors.cu:47-80): one 256-thread
// CTA per matrix, 64 KB of dynamic shared memory, raised once per device.
//
//   transition[n] = diag(alpha[n]) (I + A[n])^-1,  injection[n] = B[n] (I + A[n])^-1
//
// A, B, transition, injection: [n, 128, 128] fp32; alpha: [n, 128] fp32; all 16-byte
// aligned (the kernel reads and writes float4).
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "vdn_delta_factors.cuh"

extern "C" int ref_delta_factors(const float* A, const float* B, const float* alpha, float* transition,
                                 float* injection, int64_t n, cudaStream_t stream) {
  using namespace vdn_paper::vdn_delta_factors;
  if (n < 0 || n > 2147483647LL) return static_cast<int>(cudaErrorInvalidValue);
  if (n == 0) return 0;
  const void* ptrs[5] = {A, B, alpha, transition, injection};
  for (const void* p : ptrs)
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 16) return static_cast<int>(cudaErrorInvalidValue);
  static std::mutex mutex;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (dev < 0 || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  {
    std::lock_guard<std::mutex> lock(mutex);
    if (!configured[dev]) {
      err = cudaFuncSetAttribute(vdn_delta_factors_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kXsBytes);
      if (err != cudaSuccess) return static_cast<int>(err);
      configured[dev] = true;
    }
  }
  vdn_delta_factors_kernel<<<static_cast<unsigned>(n), kBlockSize, kXsBytes, stream>>>(A, B, alpha, transition,
                                                                                        injection);
  return static_cast<int>(cudaGetLastError());
}
