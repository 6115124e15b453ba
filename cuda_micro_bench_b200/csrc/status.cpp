// status.cpp — status strings, per-thread last error, device queries.
#include <cstdio>
#include <mutex>
#include <string>

#include "cmb_host.h"

namespace cmb {

static thread_local std::string t_last_error;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

void clear_error() { t_last_error.clear(); }

int current_sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int current_cc() {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major * 10 + minor;
}

}  // namespace cmb

extern "C" const char *cmb_status_string(int status) {
  switch (status) {
    case CMB_OK: return "CMB_OK";
    case CMB_ERR_INVALID_ARG: return "CMB_ERR_INVALID_ARG";
    case CMB_ERR_CUDA: return "CMB_ERR_CUDA";
    case CMB_ERR_TIMEOUT: return "CMB_ERR_TIMEOUT";
    case CMB_ERR_UNSUPPORTED: return "CMB_ERR_UNSUPPORTED";
    case CMB_ERR_MISMATCH: return "CMB_ERR_MISMATCH";
    case CMB_ERR_IO: return "CMB_ERR_IO";
    default: return "CMB_ERR_UNKNOWN";
  }
}

extern "C" const char *cmb_last_error(void) { return cmb::t_last_error.c_str(); }

extern "C" const char *cmb_version(void) { return "cmb_b200 0.1 (sm_100a)"; }

extern "C" int cmb_device_reset(void) {
  int dev = 0;
  CMB_CUDA_TRY(cudaGetDevice(&dev));
  cmb::p2p_release_streams(dev);
  cmb::host_copy_release_streams(dev);
  cmb::gemm_release_die_map(dev);
  CMB_CUDA_TRY(cudaDeviceReset());
  return CMB_OK;
}
