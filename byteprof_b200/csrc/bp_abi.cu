// C ABI plumbing: version, status strings, the per-thread last-error message, device checks.
#include "bp_common.cuh"

namespace bp {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

int fail(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return BP_OK;
}

int require_sm100() {
  static int cached_major[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(BP_ERR_NO_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(BP_ERR_NO_DEVICE, "device index %d out of range", dev);
  if (cached_major[dev] == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return fail(BP_ERR_NO_DEVICE, "cannot query the compute capability of device %d", dev);
    cached_major[dev] = major * 10 + minor;
  }
  if (cached_major[dev] != 100)
    return fail(BP_ERR_NO_DEVICE, "device %d is sm_%d; these kernels are built for sm_100a only", dev,
                cached_major[dev]);
  return BP_OK;
}

}  // namespace bp

extern "C" {

int bp_abi_version(void) { return 205; }

const char* bp_status_string(int status) {
  switch (status) {
    case BP_OK: return "ok";
    case BP_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BP_ERR_UNSUPPORTED: return "unsupported";
    case BP_ERR_MISALIGNED: return "misaligned";
    case BP_ERR_CUDA: return "cuda error";
    case BP_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

const char* bp_last_error(void) { return bp::g_last_error.c_str(); }

}  // extern "C"
