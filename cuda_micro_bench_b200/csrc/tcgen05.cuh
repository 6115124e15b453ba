// tcgen05.cuh — inline PTX for the 5th-generation tensor core (sm_100a):
// TMEM allocation, shared-memory matrix descriptors, instruction
// descriptors, tcgen05.mma / commit / ld, and the cluster helpers the
// 2-CTA (cta_group::2) GEMM needs.  Nothing here addresses another GPU's
// memory, and no load or commit names more than one destination CTA.
#pragma once

#include <cstdint>

namespace cmb {
namespace tc {

// ------------------------------------------------------------- cluster

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared::cta location in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ---------------------------------------------------------------- TMEM

template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t cols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     holder_smem),
                 "r"(cols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     holder_smem),
                 "r"(cols)
                 : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CG == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ------------------------------------------------------- descriptors

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzling: rows of 128 bytes, 8-row (1024-byte) swizzle
// atoms stacked along M/N.  Fields: start address >> 4 (bits 0-13), leading
// byte offset >> 4 (16-29; unused for swizzled K-major, set to 1), stride
// byte offset >> 4 = 1024 >> 4 (32-45), descriptor version 1 (46-47), base
// offset 0 (49-51, atoms 1024-byte aligned), layout 2 = SWIZZLE_128B (61-63).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  return (static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu)) | (1ull << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, dense MMA, both operands K-major, fp32 accumulate.
//   bits 4-5 D format (1 = f32); 7-9 A format; 10-12 B format
//   (kind::f16: 1 = bf16; kind::f8f6f4: 0 = e4m3); 15/16 A/B major (0 = K);
//   17-22 N >> 3; 24-28 M >> 4.
template <int M, int N, bool kFp8>
__host__ __device__ constexpr uint32_t instr_desc() {
  return (1u << 4) | ((kFp8 ? 0u : 1u) << 7) | ((kFp8 ? 0u : 1u) << 10) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- MMA

// D[tmem] (+)= A[smem] * B[smem]^T; issued by one thread.
template <int CG, bool kFp8>
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                    uint32_t idesc, uint32_t accumulate) {
  if constexpr (CG == 1 && !kFp8)
    asm volatile(
        "{ .reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  else if constexpr (CG == 1 && kFp8)
    asm volatile(
        "{ .reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  else if constexpr (CG == 2 && !kFp8)
    asm volatile(
        "{ .reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  else
    asm volatile(
        "{ .reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the mbarrier at `bar` (a shared::cluster address; a
// shared::cta address names the issuing CTA) when all tcgen05 operations
// this thread issued before have completed.
template <int CG>
__device__ __forceinline__ void commit(uint32_t bar) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                     "r"(bar)
                 : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
                     "r"(bar)
                 : "memory");
}

// ------------------------------------------------------------ TMEM -> regs

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (warp's quarter * 32 + t), columns [col, col + 32).
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------- TMA loads

// 2-D tiled load into this CTA's shared memory whose completion is counted
// on the mbarrier `bar` of CTA 0 of the pair (shared::cluster address):
// the cta_group::2 form used by both CTAs of a 2-CTA MMA pair.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *tmap, int32_t x,
                                                 int32_t y, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

}  // namespace tc
}  // namespace cmb
