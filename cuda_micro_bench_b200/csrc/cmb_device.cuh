// cmb_device.cuh — device-side helpers shared by the probe kernels (sm_100a).
//
// Inline PTX for the memory, timer, mbarrier and bulk-copy instructions the
// probes use, plus the bounded-wait rule: every spin on an mbarrier gives up
// after a deadline on %globaltimer and reports CMB_ERR_TIMEOUT instead of
// hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/cmb_b200.h"

namespace cmb {
namespace dev {

// ---------------------------------------------------------------- timers

__device__ __forceinline__ uint64_t clock64() {
  uint64_t r;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(r));
  return r;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t r;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(r));
  return r;
}

// Reads %clock64 only after `dep` is available: both predicated reads
// depend on the value, so the read cannot be hoisted above the chain that
// produced it (the reference's clockAfter64, include/timer.h:50-58).
__device__ __forceinline__ uint64_t clock64_after(uint32_t dep) {
  uint64_t r;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "setp.eq.u32 p, %1, 0;\n\t"
      "@p mov.u64 %0, %%clock64;\n\t"
      "@!p mov.u64 %0, %%clock64; }"
      : "=l"(r)
      : "r"(dep)
      : "memory");
  return r;
}

__device__ __forceinline__ uint64_t globaltimer_after(uint32_t dep) {
  uint64_t r;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "setp.eq.u32 p, %1, 0;\n\t"
      "@p mov.u64 %0, %%globaltimer;\n\t"
      "@!p mov.u64 %0, %%globaltimer; }"
      : "=l"(r)
      : "r"(dep)
      : "memory");
  return r;
}

// --------------------------------------------------------- global memory

// 16-byte streaming load: read-only path, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16-byte streaming store (evict-first).
__device__ __forceinline__ void st_stream_v4(void *p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t ld_cg_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_ca_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.global.ca.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------- mbarrier

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (shared::cluster
// address from mapa).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_cluster_acq(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Default limit for one device-side wait.  Every probe finishes its waits in
// microseconds; a wait that reaches this limit means a lost arrival.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Waits for phase `parity` of the barrier to complete.  Returns false (and
// leaves the barrier alone) once kWaitLimitNs has passed.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
#pragma unroll 1
  for (int i = 0; i < 64; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t deadline = globaltimer() + limit_ns;
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() > deadline) return false;
  }
}

__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity,
                                                          uint64_t limit_ns = kWaitLimitNs) {
#pragma unroll 1
  for (int i = 0; i < 64; ++i)
    if (mbar_try_wait_cluster_acq(bar, parity)) return true;
  const uint64_t deadline = globaltimer() + limit_ns;
#pragma unroll 1
  while (true) {
    if (mbar_try_wait_cluster_acq(bar, parity)) return true;
    if (globaltimer() > deadline) return false;
  }
}

// Records the first failure of a launch in its status word.
__device__ __forceinline__ void report_status(int *status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------- TMA (no
// cluster-wide destination form is used anywhere in this library)

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void tma_load_1d(uint32_t dst, const void *tmap, int32_t x,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.1d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2}], [%3];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, int32_t x, int32_t y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void *tmap, int32_t x,
                                                 int32_t y, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const void *tmap, int32_t x, int32_t y,
                                             uint32_t src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          tmap),
      "r"(x), "r"(y), "r"(src)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d_hint(const void *tmap, int32_t x, int32_t y,
                                                  uint32_t src, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group.L2::cache_hint"
      " [%0, {%1, %2}], [%3], %4;" ::"l"(tmap),
      "r"(x), "r"(y), "r"(src), "l"(policy)
      : "memory");
}

// Untiled bulk copies (no tensor map): global -> this CTA's shared memory,
// completion counted on `bar`; shared memory -> global, in the calling
// thread's bulk group.  Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void bulk_store(void *dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------ warp utils

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------- generators

__host__ __device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint32_t fmix32_index(uint32_t i) {
  uint32_t x = i + 0x9e3779b9u;
  x = (x ^ (x >> 16)) * 0x85ebca6bu;
  x = (x ^ (x >> 13)) * 0xc2b2ae35u;
  return x ^ (x >> 16);
}

}  // namespace dev
}  // namespace cmb
