// selftest.cu — exercises the bounded-wait rule on the device: one thread
// waits on an mbarrier phase that nothing completes, with a caller-chosen
// limit, and must come back with CMB_ERR_TIMEOUT instead of hanging.  This is
// how the probe kernels' timeout paths are tested without faulting a GPU.
#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

__global__ void k_wait_timeout(uint64_t limit_ns, int *status, uint64_t *waited_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = dev::smem_addr(&bar);
  dev::mbar_init(b, 1);  // expects one arrival that never comes
  dev::fence_mbar_init();
  const uint64_t t0 = dev::globaltimer();
  const bool ok = dev::mbar_wait_bounded(b, 0, limit_ns);
  *waited_ns = dev::globaltimer() - t0;
  dev::report_status(status, ok ? CMB_ERR_MISMATCH : CMB_ERR_TIMEOUT);
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_selftest_wait_timeout(uint64_t limit_ns, int *status, uint64_t *waited_ns,
                                         cmb_stream_t stream) {
  if (status == nullptr || waited_ns == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_selftest_wait_timeout: null output");
  if (limit_ns == 0 || limit_ns > 2000000000ull)
    return fail(CMB_ERR_INVALID_ARG, "cmb_selftest_wait_timeout: limit %llu ns not in (0, 2 s]",
                static_cast<unsigned long long>(limit_ns));
  CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  k_wait_timeout<<<1, 32, 0, stream>>>(limit_ns, status, waited_ns);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
