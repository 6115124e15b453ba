// chase.cu — dependent-load pointer chase (reference src/memory_chase.cu,
// include/memory_chase.h).
//
// The link array covers bytes/128 slots of 128 bytes; word 0 of a slot holds
// the word index of the next slot, so each hop touches a new line and one
// walk of the cycle visits every slot once.  One thread walks it; the timed
// hops are bracketed by %clock64 and %globaltimer reads that depend on the
// walk's result.
//
// Before the walk a parallel pass checks that every slot head holds a slot
// index in range, so a corrupt array ends in CMB_ERR_INVALID_ARG instead of
// an out-of-bounds load.
#include <thread>
#include <vector>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

__global__ void k_chase_validate(const uint32_t *links, size_t words, uint64_t *out) {
  const size_t slots = words / 32;
  for (size_t s = blockIdx.x * (size_t)blockDim.x + threadIdx.x; s < slots;
       s += (size_t)gridDim.x * blockDim.x) {
    uint32_t v = __ldcg(links + s * 32);
    if ((v & 31u) != 0 || v >= words) atomicExch(reinterpret_cast<unsigned long long *>(out + 3),
                                                 static_cast<unsigned long long>(CMB_ERR_INVALID_ARG));
  }
}

template <bool kBypassL1>
__device__ __forceinline__ uint32_t hop(const uint32_t *links, uint32_t idx) {
  return kBypassL1 ? dev::ld_cg_u32(links + idx) : dev::ld_ca_u32(links + idx);
}

template <bool kBypassL1>
__global__ void k_chase(const uint32_t *links, uint64_t warmup, uint64_t hops, uint64_t *out) {
  if (out[3] != 0) return;  // validation failed
  uint32_t idx = 0;
#pragma unroll 1
  for (uint64_t r = 0; r < warmup; ++r) idx = hop<kBypassL1>(links, idx);
  const uint64_t c0 = dev::clock64_after(idx);
  const uint64_t t0 = dev::globaltimer_after(idx);
  uint64_t r = 0;
#pragma unroll 1
  for (; r + 16 <= hops; r += 16) {
#pragma unroll
    for (int u = 0; u < 16; ++u) idx = hop<kBypassL1>(links, idx);
  }
#pragma unroll 1
  for (; r < hops; ++r) idx = hop<kBypassL1>(links, idx);
  const uint64_t c1 = dev::clock64_after(idx);
  const uint64_t t1 = dev::globaltimer_after(idx);
  out[0] = c1 - c0;
  out[1] = idx;
  out[2] = t1 - t0;
}

uint64_t splitmix_at(uint64_t seed, uint64_t i) { return dev::splitmix64_at(seed, i); }

}  // namespace

uint64_t splitmix64_host(uint64_t seed, uint64_t i) { return dev::splitmix64_at(seed, i); }

}  // namespace cmb

using namespace cmb;

extern "C" int cmb_chase_build_links(uint32_t *host_links, size_t bytes, uint64_t seed) {
  if (host_links == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_chase_build_links: null");
  if (bytes < 128 || bytes % 128 != 0)
    return fail(CMB_ERR_INVALID_ARG, "cmb_chase_build_links: bytes %zu not a multiple of 128",
                bytes);
  if (bytes / 4 > 0xffffffffull)
    return fail(CMB_ERR_INVALID_ARG, "cmb_chase_build_links: %zu bytes exceed 32-bit indices",
                bytes);
  const size_t words = bytes / 4, slots = bytes / 128;
  // Padding words: fmix32 of the word index (include/memory_chase.h:128-133),
  // filled by all host threads.
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (nt > 64) nt = 64;
  if (words < (1u << 20)) nt = 1;
  std::vector<std::thread> pool;
  for (unsigned t = 0; t < nt; ++t)
    pool.emplace_back([=] {
      size_t a = words * t / nt, b = words * (t + 1) / nt;
      for (size_t w = a; w < b; ++w) host_links[w] = dev::fmix32_index(static_cast<uint32_t>(w));
    });
  for (auto &th : pool) th.join();
  // Sattolo's algorithm gives a uniformly random single cycle: for i from
  // slots-1 down to 1, exchange order[i] with order[j], j uniform in [0, i),
  // j drawn from SplitMix64 output (slots-1-i) by a 64x64->128 multiply.
  std::vector<uint32_t> next(slots);
  for (size_t s = 0; s < slots; ++s) next[s] = static_cast<uint32_t>(s);
  uint64_t draw = 0;
  for (size_t i = slots - 1; i >= 1; --i, ++draw) {
    const uint64_t r = splitmix_at(seed, draw);
    const size_t j = static_cast<size_t>((static_cast<unsigned __int128>(r) * i) >> 64);
    std::swap(next[i], next[j]);
  }
  for (size_t s = 0; s < slots; ++s) host_links[s * 32] = next[s] * 32u;
  return CMB_OK;
}

extern "C" int cmb_chase_host_walk(const uint32_t *host_links, size_t words, uint64_t hops,
                                   uint32_t *out_index) {
  if (host_links == nullptr || out_index == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_chase_host_walk: null pointer");
  uint32_t idx = 0;
  for (uint64_t h = 0; h < hops; ++h) {
    if (idx >= words)
      return fail(CMB_ERR_INVALID_ARG, "cmb_chase_host_walk: index %u out of %zu words at hop %llu",
                  idx, words, static_cast<unsigned long long>(h));
    idx = host_links[idx];
  }
  *out_index = idx;
  return CMB_OK;
}

extern "C" int cmb_chase_run(const uint32_t *links, size_t words, uint64_t warmup, uint64_t hops,
                             int bypass_l1, uint64_t *out, cmb_stream_t stream) {
  if (links == nullptr || out == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_chase_run: null links or out");
  if (words < 32 || words % 32 != 0 || words > 0xffffffffull)
    return fail(CMB_ERR_INVALID_ARG, "cmb_chase_run: words %zu must be a multiple of 32 in "
                "[32, 2^32)", words);
  CMB_CUDA_TRY(cudaMemsetAsync(out, 0, 4 * sizeof(uint64_t), stream));
  const size_t slots = words / 32;
  size_t grid = (slots + 255) / 256;
  const size_t cap = static_cast<size_t>(current_sm_count()) * 8;
  if (grid > cap) grid = cap;
  k_chase_validate<<<static_cast<int>(grid), 256, 0, stream>>>(links, words, out);
  CMB_LAUNCH_CHECK();
  if (bypass_l1)
    k_chase<true><<<1, 1, 0, stream>>>(links, warmup, hops, out);
  else
    k_chase<false><<<1, 1, 0, stream>>>(links, warmup, hops, out);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
