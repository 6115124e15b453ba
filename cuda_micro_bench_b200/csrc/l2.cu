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

// Bulk-copy form: the same exact word sum with the bytes brought into shared
// memory by cp.async.bulk (the TMA unit) instead of register loads.  Each
// warp owns a kL2BulkStages-deep ring of 8 KiB chunks: lane 0 issues the
// loads, all 32 lanes add the words of each landed chunk, then lane 0
// refills the stage.  One issuing thread's bulk copies reach only part of
// what L2 delivers to an SM, so twelve warps per SM issue side by side (on
// B200, 8 MiB resident: 4 warps x 3 stages of 16 KiB 16.8 TB/s, 12 x 2 of
// 8 KiB 21.9, 24 x 1 of 8 KiB 22.5; register loads 12.8).  Warp w of W takes
// units w, w + W, ...; unit u reads chunk u % nchunk, so after
// passes * nchunk units every chunk was read `passes` times.
constexpr int kL2BulkWarps = 12;
constexpr int kL2BulkStages = 2;
constexpr uint32_t kL2Chunk = 8192;

__global__ void __launch_bounds__(32 * kL2BulkWarps, 1)
    k_l2_read_bulk(const char *__restrict__ data, size_t nchunk, int passes,
                   unsigned long long *sum, int *status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kL2BulkWarps][kL2BulkStages];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *ring = smem + (size_t)warp * kL2BulkStages * kL2Chunk;
  const size_t W = (size_t)gridDim.x * kL2BulkWarps;
  const size_t w = (size_t)blockIdx.x * kL2BulkWarps + warp;
  const size_t units = nchunk * (size_t)passes;
  const size_t mine = units > w ? (units - 1 - w) / W + 1 : 0;
  if (lane == 0)
    for (int s = 0; s < kL2BulkStages; ++s) dev::mbar_init(dev::smem_addr(&full[warp][s]), 1);
  dev::fence_mbar_init();
  __syncwarp();
  const auto issue = [&](size_t k) {  // lane 0: load unit k of this warp into its stage
    const int s = static_cast<int>(k % kL2BulkStages);
    const uint32_t bar = dev::smem_addr(&full[warp][s]);
    const size_t chunk = (w + k * W) % nchunk;
    dev::mbar_arrive_expect_tx(bar, kL2Chunk);
    dev::bulk_load(dev::smem_addr(ring + (size_t)s * kL2Chunk), data + chunk * kL2Chunk,
                   kL2Chunk, bar);
  };
  if (lane == 0)
    for (size_t k = 0; k < mine && k < (size_t)kL2BulkStages; ++k) issue(k);
  unsigned long long acc = 0;
  size_t k = 0;
  for (; k < mine; ++k) {
    const int s = static_cast<int>(k % kL2BulkStages);
    // every lane waits (acquire) before reading the chunk
    const bool ok = dev::mbar_wait_bounded(dev::smem_addr(&full[warp][s]),
                                           static_cast<uint32_t>(k / kL2BulkStages) & 1);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) dev::report_status(status, CMB_ERR_TIMEOUT);
      break;
    }
    const uint4 *v = reinterpret_cast<const uint4 *>(ring + (size_t)s * kL2Chunk);
#pragma unroll 8
    for (int i = lane; i < (int)(kL2Chunk / 16); i += 32) {
      const uint4 x = v[i];
      acc += (unsigned long long)x.x + x.y + x.z + x.w;
    }
    __syncwarp();
    if (lane == 0 && k + kL2BulkStages < mine) issue(k + kL2BulkStages);
  }
  // After a failed wait: wait (bounded) for the loads still writing the ring.
  if (lane == 0)
    for (size_t j = k; j < mine && j < k + kL2BulkStages; ++j)
      if (!dev::mbar_wait_bounded(dev::smem_addr(&full[warp][j % kL2BulkStages]),
                                  static_cast<uint32_t>(j / kL2BulkStages) & 1, 100000000ull))
        break;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) atomicAdd(sum, acc);
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_l2_read_bulk(const void *buf, size_t bytes, int passes, unsigned long long *sum,
                                int *status, cmb_stream_t stream) {
  if (buf == nullptr || sum == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_l2_read_bulk: null pointer");
  if (bytes == 0 || bytes % kL2Chunk != 0 || (reinterpret_cast<uintptr_t>(buf) & 15))
    return fail(CMB_ERR_INVALID_ARG, "cmb_l2_read_bulk: bytes must be a positive multiple of "
                "8 KiB, 16-byte aligned");
  if (passes < 1) return fail(CMB_ERR_INVALID_ARG, "cmb_l2_read_bulk: passes < 1");
  const size_t smem = (size_t)kL2BulkWarps * kL2BulkStages * kL2Chunk;
  CMB_CUDA_TRY(cudaFuncSetAttribute(k_l2_read_bulk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  CMB_CUDA_TRY(cudaMemsetAsync(sum, 0, sizeof(unsigned long long), stream));
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  k_l2_read_bulk<<<current_sm_count(), 32 * kL2BulkWarps, smem, stream>>>(
      static_cast<const char *>(buf), bytes / kL2Chunk, passes, sum, status);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

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
