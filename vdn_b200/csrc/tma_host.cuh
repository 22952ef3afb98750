// Host-side TMA tensor-map encoding through the driver entry point (no -lcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace vdn {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// Tiled map with the given swizzle mode (the store maps of the bulk-store epilogues
// use 64-byte swizzle: 32 x 64-byte pieces).
inline int encode_map_swizzle(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                              const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                              CUtensorMapSwizzle swizzle) {
  auto fn = tensor_map_encoder();
  if (!fn) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VDN_OK;
}

// Tiled map with 128B swizzle.  dims / box innermost first; strides_bytes has
// rank-1 entries (the strides of dims 1..rank-1).
inline int encode_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  auto fn = tensor_map_encoder();
  if (!fn) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VDN_ERR_RUNTIME, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VDN_OK;
}

}  // namespace vdn
