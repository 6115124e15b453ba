// l2.cu — L2 aggregate read bandwidth (reference src/memory_more.cu:66-85,
// 201-234): every SM streams 16-byte .cg loads (L1 bypassed) over a buffer
// that stays resident in L2, `passes` times.  Each thread adds the 32-bit
// words it loads into a 64-bit integer sum, so the result is exact:
// passes * (sum of the buffer's words) modulo 2^64.
#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

constexpr int kL2Threads = 256;

__global__ void __launch_bounds__(kL2Threads) k_l2_read(const uint4 *__restrict__ data, size_t nvec,
                                                        int passes, unsigned long long *sum) {
  unsigned long long acc = 0;
  const size_t stride = (size_t)gridDim.x * kL2Threads;
  const size_t t = blockIdx.x * (size_t)kL2Threads + threadIdx.x;
#pragma unroll 1
  for (int p = 0; p < passes; ++p) {
    // grid-stride: every element once per pass, four loads in flight
    for (size_t i = t; i < nvec; i += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const size_t idx = i + u * stride;
        if (idx < nvec)
          asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w)
                       : "l"(data + idx));
        else
          v[u] = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) acc += (unsigned long long)v[u].x + v[u].y + v[u].z + v[u].w;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(sum, acc);
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_l2_read(const void *buf, size_t bytes, int passes, int ctas,
                           unsigned long long *sum, cmb_stream_t stream) {
  if (buf == nullptr || sum == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_l2_read: null pointer");
  if (bytes < 16 || bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(buf) & 15))
    return fail(CMB_ERR_INVALID_ARG, "cmb_l2_read: bytes must be a positive multiple of 16, "
                "16-byte aligned");
  if (passes < 1) return fail(CMB_ERR_INVALID_ARG, "cmb_l2_read: passes < 1");
  if (ctas <= 0) ctas = current_sm_count() * 4;
  CMB_CUDA_TRY(cudaMemsetAsync(sum, 0, sizeof(unsigned long long), stream));
  k_l2_read<<<ctas, kL2Threads, 0, stream>>>(static_cast<const uint4 *>(buf), bytes / 16, passes,
                                              sum);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
