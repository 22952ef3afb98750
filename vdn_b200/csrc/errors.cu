// Thread-local last-error message and library metadata entry points.
#include "common.cuh"

#include <string.h>

namespace vdn {

static thread_local char g_last_error[1024] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = '\0'; }

}  // namespace vdn

extern "C" {

const char* vdn_last_error(void) { return vdn::g_last_error; }

int vdn_abi_version(void) { return VDN_ABI_VERSION; }

int vdn_device_supported(int device, int* supported) {
  if (!supported) return vdn::set_error(VDN_ERR_VALUE, "supported must not be null");
  int major = 0, minor = 0;
  VDN_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  VDN_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  *supported = (major == 10 && minor == 0) ? 1 : 0;
  return VDN_OK;
}

}  // extern "C"
