// verify.cu — device-side result checks the probe sections use: byte
// comparison of two buffers (copies and tile moves must be bit-exact).
#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

__global__ void k_count_mismatch(const uint4 *__restrict__ a, const uint4 *__restrict__ b,
                                 size_t nvec, const uint8_t *__restrict__ ta,
                                 const uint8_t *__restrict__ tb, size_t tail,
                                 unsigned long long *count) {
  unsigned long long local = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nvec;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint4 x = __ldg(a + i), y = __ldg(b + i);
    local += (x.x != y.x) + (x.y != y.y) + (x.z != y.z) + (x.w != y.w);
  }
  if (blockIdx.x == 0)
    for (size_t i = threadIdx.x; i < tail; i += blockDim.x) local += (ta[i] != tb[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if ((threadIdx.x & 31) == 0 && local != 0) atomicAdd(count, local);
}

__global__ void k_count_mismatch_bytes(const uint8_t *a, const uint8_t *b, size_t n,
                                       unsigned long long *count) {
  unsigned long long local = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    local += (a[i] != b[i]);
  if (local != 0) atomicAdd(count, local);
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_compare_bytes(const void *a, const void *b, size_t bytes,
                                 unsigned long long *mismatches, cmb_stream_t stream) {
  if (mismatches == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_compare_bytes: null output");
  if (bytes > 0 && (a == nullptr || b == nullptr))
    return fail(CMB_ERR_INVALID_ARG, "cmb_compare_bytes: null buffer");
  CMB_CUDA_TRY(cudaMemsetAsync(mismatches, 0, sizeof(unsigned long long), stream));
  if (bytes == 0) return CMB_OK;
  const int grid = current_sm_count() * 4;
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0) {
    const size_t nvec = bytes / 16;
    const uint8_t *ta = static_cast<const uint8_t *>(a) + nvec * 16;
    const uint8_t *tb = static_cast<const uint8_t *>(b) + nvec * 16;
    k_count_mismatch<<<grid, 256, 0, stream>>>(static_cast<const uint4 *>(a),
                                               static_cast<const uint4 *>(b), nvec, ta, tb,
                                               bytes - nvec * 16, mismatches);
  } else {
    k_count_mismatch_bytes<<<grid, 256, 0, stream>>>(static_cast<const uint8_t *>(a),
                                                     static_cast<const uint8_t *>(b), bytes,
                                                     mismatches);
  }
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
