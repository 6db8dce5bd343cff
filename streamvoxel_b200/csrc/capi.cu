// C-ABI plumbing: error text, version, device check.
#include "common.cuh"

namespace svx {

static thread_local std::string g_error;

void set_error(const std::string& text) { g_error = text; }

int fail(int status, const std::string& text) {
  g_error = text;
  return status;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SVX_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return SVX_OK;
}

}  // namespace svx

extern "C" const char* svx_last_error(void) { return svx::g_error.c_str(); }

extern "C" int svx_version(void) { return 1; }

extern "C" int svx_device_supported(void) {
  int device = 0, major = 0, minor = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return 0;
  return major == 10 && minor == 0;
}
