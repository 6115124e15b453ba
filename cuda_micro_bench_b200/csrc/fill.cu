// fill.cu — seeded input generators.  Counter-based (output i depends only on
// the seed and i), so any grid produces the same array and the CPU oracle can
// regenerate the integer and uniform streams bit for bit.
#include <cuda_bf16.h>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

constexpr int kFillThreads = 256;

int fill_grid(size_t n) {
  size_t want = (n + kFillThreads - 1) / kFillThreads;
  size_t cap = static_cast<size_t>(current_sm_count()) * 8;
  if (want > cap) want = cap;
  return want == 0 ? 1 : static_cast<int>(want);
}

// Reference kernel_init_stream (src/mem_global.cu:5-12), 64-bit index.
__global__ void k_fill_hash_u32(uint32_t *dst, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = dev::fmix32_index(static_cast<uint32_t>(i));
}

__global__ void k_fill_uniform_f32(float *dst, size_t n, uint64_t seed) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    uint32_t u = static_cast<uint32_t>(dev::splitmix64_at(seed, i) >> 40);
    dst[i] = __fsub_rn(__fmul_rn(static_cast<float>(u), 0x1p-23f), 1.0f);
  }
}

__global__ void k_fill_bytes(uint8_t *dst, size_t n, uint64_t seed) {
  const size_t words = n / 8;
  uint64_t *d64 = reinterpret_cast<uint64_t *>(dst);
  const bool aligned = (reinterpret_cast<uintptr_t>(dst) & 7) == 0;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (aligned) {
    for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < words; w += stride)
      d64[w] = dev::splitmix64_at(seed, w);
    for (size_t i = words * 8 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
      dst[i] = static_cast<uint8_t>(dev::splitmix64_at(seed, i >> 3) >> (8 * (i & 7)));
  } else {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride)
      dst[i] = static_cast<uint8_t>(dev::splitmix64_at(seed, i >> 3) >> (8 * (i & 7)));
  }
}

// Box-Muller: output w of SplitMix64 gives values 2w and 2w+1.  u1 in
// (0, 1] from the top 24 bits, u2 in [0, 1) from the next 24 bits.
__global__ void k_fill_normal_bf16(__nv_bfloat16 *dst, size_t n, uint64_t seed, float scale) {
  const size_t pairs = (n + 1) / 2;
  for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < pairs;
       w += (size_t)gridDim.x * blockDim.x) {
    uint64_t r = dev::splitmix64_at(seed, w);
    float u1 = (static_cast<float>(static_cast<uint32_t>(r >> 40)) + 1.0f) * 0x1p-24f;
    float u2 = static_cast<float>(static_cast<uint32_t>(r >> 16) & 0xffffffu) * 0x1p-24f;
    float rad = sqrtf(-2.0f * logf(u1));
    float s, c;
    sincospif(2.0f * u2, &s, &c);
    dst[2 * w] = __float2bfloat16_rn(scale * rad * c);
    if (2 * w + 1 < n) dst[2 * w + 1] = __float2bfloat16_rn(scale * rad * s);
  }
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_fill_hash_u32(uint32_t *dst, size_t n, cmb_stream_t stream) {
  if (n == 0) return CMB_OK;
  if (dst == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_fill_hash_u32: null dst");
  k_fill_hash_u32<<<fill_grid(n), kFillThreads, 0, stream>>>(dst, n);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

extern "C" int cmb_fill_uniform_f32(float *dst, size_t n, uint64_t seed, cmb_stream_t stream) {
  if (n == 0) return CMB_OK;
  if (dst == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_fill_uniform_f32: null dst");
  k_fill_uniform_f32<<<fill_grid(n), kFillThreads, 0, stream>>>(dst, n, seed);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

extern "C" int cmb_fill_bytes(uint8_t *dst, size_t n, uint64_t seed, cmb_stream_t stream) {
  if (n == 0) return CMB_OK;
  if (dst == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_fill_bytes: null dst");
  k_fill_bytes<<<fill_grid(n / 8 + 1), kFillThreads, 0, stream>>>(dst, n, seed);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

extern "C" int cmb_fill_normal_bf16(uint16_t *dst, size_t n, uint64_t seed, float scale,
                                    cmb_stream_t stream) {
  if (n == 0) return CMB_OK;
  if (dst == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_fill_normal_bf16: null dst");
  k_fill_normal_bf16<<<fill_grid((n + 1) / 2), kFillThreads, 0, stream>>>(
      reinterpret_cast<__nv_bfloat16 *>(dst), n, seed, scale);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
