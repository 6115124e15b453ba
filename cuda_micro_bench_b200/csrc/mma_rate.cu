// mma_rate.cu — tensor-pipe ceiling with shared-memory operands: the
// tcgen05 counterpart of the reference's register-only mma.sync throughput
// kernels (src/tensor_core.cu:41-64, src/tensor_core_extended.cu:227-250),
// which multiply constant 1.0 operands and keep the sum.
//
// Each CTA fills one 128 x (128 bytes) A tile and one 256 x (128 bytes) B tile
// of ones in shared memory, then one thread issues `iters` rounds of four
// tcgen05.mma (M=128, N=256, 32 bytes of K each) into one TMEM accumulator
// with no memory traffic, so the launch time is the tensor pipe's issue and
// execute rate.  Every accumulator element ends at iters * 4 * K_instr
// (K_instr = 16 for bf16, 32 for e4m3), which the epilogue checks and
// writes (one value per row) so the result is observable.
#include "cmb_device.cuh"
#include "cmb_host.h"
#include "tcgen05.cuh"

namespace cmb {
namespace {

constexpr int kRateThreads = 128;
constexpr int kRateABytes = 128 * 128, kRateBBytes = 256 * 128;

template <bool kFp8>
__global__ void __launch_bounds__(kRateThreads, 1)
    k_mma_rate(int iters, float *out, uint64_t *cycles, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *tile = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_holder;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ones: bf16 1.0 = 0x3F80, e4m3 1.0 = 0x38 (layout-independent).
  const uint32_t one4 = kFp8 ? 0x38383838u : 0x3F803F80u;
  const uint4 v = make_uint4(one4, one4, one4, one4);
  for (int i = threadIdx.x; i < (kRateABytes + kRateBBytes) / 16; i += kRateThreads)
    reinterpret_cast<uint4 *>(tile)[i] = v;
  dev::fence_proxy_async_smem();  // generic-proxy writes -> tensor core reads
  if (threadIdx.x == 0) {
    dev::mbar_init(dev::smem_addr(&done), 1);
    dev::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc<1>(dev::smem_addr(&tmem_holder), 256);
    tc::tmem_relinquish<1>();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_holder;

  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = tc::instr_desc<128, 256, kFp8>();
    const uint32_t a = dev::smem_addr(tile);
    const uint64_t da = tc::sw128_kmajor_desc(a), db = tc::sw128_kmajor_desc(a + kRateABytes);
    const uint64_t t0 = dev::clock64();
#pragma unroll 1
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) tc::mma<1, kFp8>(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
    }
    tc::commit<1>(dev::smem_addr(&done));
    if (!dev::mbar_wait_bounded(dev::smem_addr(&done), 0))
      dev::report_status(status, CMB_ERR_TIMEOUT);
    const uint64_t t1 = dev::clock64();
    if (cycles != nullptr) cycles[blockIdx.x] = t1 - t0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  // Each warp reads its 32 TMEM lanes (rows), columns 0-31.
  uint32_t r[32];
  tc::ld_32x32b_x32(tmem + (static_cast<uint32_t>(warp * 32) << 16), r);
  tc::wait_ld();
  const float expect = static_cast<float>(iters) * 4.0f * (kFp8 ? 32.0f : 16.0f);
  bool ok = true;
#pragma unroll
  for (int i = 0; i < 32; ++i) ok &= (__uint_as_float(r[i]) == expect);
  if (!ok) dev::report_status(status, CMB_ERR_MISMATCH);
  out[(size_t)blockIdx.x * 128 + warp * 32 + lane] = __uint_as_float(r[0]);

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc<1>(tmem, 256);
  }
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_mma_rate(int fp8, int iters, int ctas, float *out, uint64_t *cycles,
                            int *status, cmb_stream_t stream) {
  if (out == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_mma_rate: null out");
  if (iters < 1 || iters > (1 << 20))
    return fail(CMB_ERR_INVALID_ARG, "cmb_mma_rate: iters %d not in [1, 2^20]", iters);
  if (ctas < 1 || ctas > 65535) return fail(CMB_ERR_INVALID_ARG, "cmb_mma_rate: ctas %d", ctas);
  if (current_cc() != 100)
    return fail(CMB_ERR_UNSUPPORTED, "cmb_mma_rate: needs an sm_100 device (cc %d)", current_cc());
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  // 120 KiB of dynamic shared memory (48 KiB used) keeps one CTA per SM, so
  // each CTA owns its SM's tensor core and TMEM.
  const size_t smem = 120 * 1024;
  if (fp8) {
    CMB_CUDA_TRY(cudaFuncSetAttribute(k_mma_rate<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
    k_mma_rate<true><<<ctas, kRateThreads, smem, stream>>>(iters, out, cycles, status);
  } else {
    CMB_CUDA_TRY(cudaFuncSetAttribute(k_mma_rate<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
    k_mma_rate<false><<<ctas, kRateThreads, smem, stream>>>(iters, out, cycles, status);
  }
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
