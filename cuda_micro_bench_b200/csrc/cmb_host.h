// cmb_host.h — host-side error handling shared by the C ABI entry points.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "../../include/cmb_b200.h"

namespace cmb {

// Records a one-line reason for the calling thread and returns `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
// Clears the calling thread's last error.
void clear_error();

// Number of SMs of the current device (cached per device).
int current_sm_count();
// Compute capability major*10+minor of the current device.
int current_cc();

// Output i of the SplitMix64 stream of `seed`, on the host (the generator
// of the cmb_fill_* kernels).
uint64_t splitmix64_host(uint64_t seed, uint64_t i);

// Release the library's cached streams and events of device `dev`
// (cmb_device_reset calls these before resetting the device).
void p2p_release_streams(int dev);
void host_copy_release_streams(int dev);
// Forget the die map installed for device `dev` (its device copy is gone
// after a reset).
void gemm_release_die_map(int dev);

// The source file's name without its directories (error messages name the
// file, not the machine it was built on).
inline const char *source_name(const char *path) {
  const char *base = path;
  for (const char *p = path; *p != '\0'; ++p)
    if (*p == '/') base = p + 1;
  return base;
}

}  // namespace cmb

#define CMB_CUDA_TRY(call)                                                              \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return ::cmb::fail(CMB_ERR_CUDA, "%s:%d: %s: %s", ::cmb::source_name(__FILE__),   \
                         __LINE__, #call, cudaGetErrorString(e_));                      \
  } while (0)

// Checks the launch that was just enqueued.
#define CMB_LAUNCH_CHECK() CMB_CUDA_TRY(cudaGetLastError())
