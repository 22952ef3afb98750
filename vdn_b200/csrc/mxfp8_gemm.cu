// Block-scaled MXFP8 GEMM (tcgen05 kind::mxf8f6f4) -- entry point placeholder.
#include "common.cuh"

extern "C" int vdn_mxfp8_gemm(const uint8_t*, const uint8_t*, const uint8_t*, const uint8_t*,
                              const void*, int64_t, int64_t, int64_t, int64_t, int64_t, void*,
                              int64_t, cudaStream_t) {
  return vdn::set_error(VDN_ERR_RUNTIME, "vdn_mxfp8_gemm is not built yet");
}
