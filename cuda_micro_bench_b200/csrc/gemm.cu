// gemm.cu — tcgen05 dense GEMM probes, BF16 and FP8 E4M3 (the tensor-core
// probes of the reference, src/tensor_core.cu and
// src/tensor_core_extended.cu, re-targeted from register-only mma.sync
// chains to a full GEMM on the 5th-generation tensor core).
//
// C[M x N] (fp32, row-major) = scale * A[M x K] * B[N x K]^T, A and B
// K-major ("row.col", src/tensor_core_extended.cu:116).
//
// Structure (one CTA per SM, persistent, 192 threads; 320 with the held
// epilogue below):
//   warp 0      TMA producer: 128-byte-swizzled K-major tiles of A and B
//               into a STAGES-deep shared-memory ring (full/empty mbarriers)
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma for each 128-byte K slice (4 instructions of
//               K = 32 bytes), tcgen05.commit frees the smem stage and, after
//               the last K block, marks the accumulator full
//   warps 2-5   epilogue: tcgen05.ld 32x32b from the accumulator, scale,
//               then either a 32 x 32 fp32 box per warp staged in swizzled
//               shared memory and written by a tiled TMA store (default), or
//               direct streaming stores (rows not TMA-addressable); two TMEM
//               accumulators (2 x 256 columns) let the epilogue of tile j
//               overlap the MMAs of tile j+1.
// CG = 1: tile 128 x 256 per CTA (cta_group::1, MMA M=128 N=256).
// CG = 2: a cluster of two CTAs computes a 256 x (256 * NSUB) tile with
//   cta_group::2 MMAs (M=256 N=256) issued by CTA 0; each CTA loads its own
//   128 rows of A and 128 rows of each N=256 slice of B, the loads of both
//   CTAs complete on CTA 0's full barrier, and CTA 0 commits to both CTAs'
//   barriers one address at a time.  NSUB = 2 (the default) issues two MMAs
//   per K slice into all 512 TMEM columns: a quarter fewer bytes loaded per
//   FLOP than 256 x 256 tiles (on B200 the load savings win: ~1.5 PFLOP/s
//   bf16 against ~1.2 for 256 x 256), but no second accumulator for the
//   epilogue to drain while the next tile runs.  With 8 epilogue warps the
//   drain is split instead: each warp loads 128 columns of one N=256 half
//   into registers and hands that half back before storing it, and the MMA
//   issuer starts the next tile on half 0 over the stages already loaded
//   while half 1 drains ("held" epilogue).
// Tile order: persistent clusters walk the tiles in raster groups of group_m
// tile rows.  With a die map installed (cmb_gemm_set_sm_die_map) the tiles
// are cut into two contiguous ranges, one per die of the B200 in proportion
// to its SMs, and each cluster works in the range of the die it runs on, so
// the operand lines one die reads are less often also read by the other die
// (fewer die-to-die crossings and L2 reads).  A cluster claims a slot of its
// die's range with an atomic counter, or a slot of the other range when its
// own are taken; there are as many slots as clusters, so every tile is
// computed once whatever the map says or where the clusters land.  The last
// cluster to claim resets the counters for the next launch.
// All waits are bounded; a wait that gives up reports CMB_ERR_TIMEOUT in
// `status` and every role drains and leaves.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <atomic>
#include <cmath>
#include <mutex>

#include "cmb_device.cuh"
#include "cmb_host.h"
#include "tcgen05.cuh"

namespace cmb {

int make_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t rows,
                 uint64_t cols, uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols,
                 CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo);

// Die (0 or 1) of the SM with each %smid on this device, written by
// cmb_gemm_set_sm_die_map.  Every device holds its own copy.
__device__ uint8_t g_sm_die[CMB_DIE_MAP_IDS];
// Slot-claim counters of the die-split tile order: per launch slot, claims
// made on die 0 and die 1 and the number of clusters done claiming.  Zero
// between launches.
constexpr int kClaimSlots = 64;
__device__ unsigned g_tile_claims[kClaimSlots][4];

namespace {

template <int CG, bool kFp8, int STAGES, bool kTmaEpi, int NSUB, int EPIW>
struct GemmCfg {
  static constexpr int kThreads = 64 + 32 * EPIW;
  static constexpr int kBmCta = 128;                 // A rows per CTA
  static constexpr int kBn = 256;                    // MMA N
  static constexpr int kTileN = kBn * NSUB;          // output columns per tile
  static constexpr int kBnCta = kBn / CG;            // B rows per N=256 sub-tile per CTA
  static constexpr int kKBytes = 128;                // K bytes per stage (one swizzle row)
  static constexpr int kElem = kFp8 ? 1 : 2;
  static constexpr int kBk = kKBytes / kElem;        // K elements per stage
  static constexpr int kMmaPerStage = 4;             // 32 bytes of K per instruction
  static constexpr int kABytes = kBmCta * kKBytes;   // 16 KiB
  static constexpr int kBSubBytes = kBnCta * kKBytes;  // 32 KiB (CG=1) / 16 KiB (CG=2)
  static constexpr int kBBytes = NSUB * kBSubBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = STAGES;
  static constexpr int kTileM = kBmCta * CG;         // output rows per tile
  static constexpr int kTmemCols = 512;              // all of TMEM
  // 256-column tiles keep two accumulators (the epilogue of one tile
  // overlaps the MMAs of the next); 512-column tiles use all 512 columns.
  static constexpr int kAccBufs = 2 / NSUB;
  // 512-column tiles with 8 epilogue warps drain each N=256 half of the
  // accumulator through registers (128 columns per warp) and hand that half
  // back before storing it, so the next tile's MMAs into it can start.
  static constexpr bool kHeld = NSUB == 2 && EPIW == 8;
  // TMA-store epilogue: 32 x 32 fp32 staging boxes, two per warp (one in the
  // held mode, which keeps its data in registers instead).
  static constexpr int kEpiBoxBytes = 32 * 32 * 4;
  static constexpr int kEpiBoxes = kHeld ? 1 : 2;
  static constexpr int kEpiBytes = kTmaEpi ? EPIW * kEpiBoxes * kEpiBoxBytes : 0;
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + kEpiBytes + 1024;
  static constexpr uint32_t kIdesc = tc::instr_desc<kTileM, kBn, kFp8>();
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int &tm,
                                            int &tn) {
  // Grouped raster: group_m tile rows advance together along N, so the CTAs
  // working at the same time share A rows and B columns in L2.
  const int per_group = group_m * tiles_n;
  const int g = t / per_group;
  const int first = g * group_m;
  const int gsize = min(tiles_m - first, group_m);
  const int r = t - g * per_group;
  tm = first + r % gsize;
  tn = r / gsize;
}

// Two floats rounded to bf16 (nearest even), `lo` in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void st_cs_u4(void *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.cs.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_cs_f4(float *p, float a, float b, float c, float d) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// kBf16Out: C is bf16 (each fp32 accumulator scaled, then rounded to
// nearest even); held-epilogue configurations only.
template <int CG, bool kFp8, int STAGES, bool kTmaEpi, int NSUB, int EPIW, bool kBf16Out = false>
__global__ void __launch_bounds__(64 + 32 * EPIW, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmC, void *__restrict__ Cv, int M, int N, int K,
           const float *scale_a, const float *scale_b, int group_m, int die_pairs0,
           int claim_slot, int *status) {
  using Cfg = GemmCfg<CG, kFp8, STAGES, kTmaEpi, NSUB, EPIW>;
  static_assert(!kBf16Out || Cfg::kHeld, "bf16 output needs the held epilogue");
  float *const C = static_cast<float *>(Cv);
  __nv_bfloat16 *const Cb = static_cast<__nv_bfloat16 *>(Cv);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[Cfg::kStages], empty[Cfg::kStages];
  __shared__ __align__(8) uint64_t tfull[2], tempty[2], mma_done;
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? tc::cluster_ctarank() : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      dev::mbar_init(dev::smem_addr(&full[s]), 1);
      dev::mbar_init(dev::smem_addr(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      dev::mbar_init(dev::smem_addr(&tfull[a]), 1);
      dev::mbar_init(dev::smem_addr(&tempty[a]), EPIW * CG);
    }
    dev::mbar_init(dev::smem_addr(&mma_done), 1);
    abort_flag = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&tmA);
    dev::tma_prefetch_desc(&tmB);
    if constexpr (kTmaEpi) dev::tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tc::tmem_alloc<CG>(dev::smem_addr(&tmem_holder), Cfg::kTmemCols);
    tc::tmem_relinquish<CG>();
  }
  const int tiles_m = (M + Cfg::kTileM - 1) / Cfg::kTileM;
  const int tiles_n = (N + Cfg::kTileN - 1) / Cfg::kTileN;
  const int tiles = tiles_m * tiles_n;
  // This cluster's tiles: t_first, t_first + t_step, ... below t_end.  CTA 0
  // decides and writes the three numbers into both CTAs' shared memory
  // before the cluster barrier below.
  __shared__ int tile_seq[3];
  if (threadIdx.x == 0 && rank == 0) {
    const int nclusters = gridDim.x / CG;
    int first = blockIdx.x / CG, step = nclusters, end = tiles;
    if (die_pairs0 >= 0) {
      uint32_t sm;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
      const int pairs[2] = {die_pairs0, nclusters - die_pairs0};
      unsigned *claims = g_tile_claims[claim_slot];
      int d = sm < CMB_DIE_MAP_IDS ? (g_sm_die[sm] & 1) : 0;
      int slot = static_cast<int>(atomicAdd(&claims[d], 1u));
      if (slot >= pairs[d]) {
        d ^= 1;
        slot = static_cast<int>(atomicAdd(&claims[d], 1u));
      }
      __threadfence();
      if (atomicAdd(&claims[2], 1u) == static_cast<unsigned>(nclusters - 1)) {
        // every cluster has claimed: leave the counters at zero
        __threadfence();
        atomicExch(&claims[0], 0u);
        atomicExch(&claims[1], 0u);
        atomicExch(&claims[2], 0u);
      }
      const int split = static_cast<int>(static_cast<long long>(tiles) * pairs[0] / nclusters);
      if (slot < pairs[d]) {
        first = (d == 0 ? 0 : split) + slot;
        step = pairs[d];
        end = d == 0 ? split : tiles;
      } else {  // no slot left: only if the counters were not at zero
        dev::report_status(status, CMB_ERR_MISMATCH);
        first = tiles;
      }
    }
    tile_seq[0] = first;
    tile_seq[1] = step;
    tile_seq[2] = end;
    if constexpr (CG == 2) {
      const int v[3] = {first, step, end};
      for (int i = 0; i < 3; ++i)
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(
                         tc::map_to_cta(dev::smem_addr(&tile_seq[i]), 1)),
                     "r"(v[i])
                     : "memory");
    }
  }
  tc::fence_before_sync();
  if constexpr (CG == 2) tc::cluster_sync();
  else __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem_base = tmem_holder;
  const int t_first = tile_seq[0], t_step = tile_seq[1], t_end = tile_seq[2];
  const int kblocks = (K + Cfg::kBk - 1) / Cfg::kBk;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int it = 0;
      bool ok = true;
      for (int t = t_first; t < t_end && ok; t += t_step) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, group_m, tm, tn);
        const int a_row = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kBmCta;
        const int b_row = tn * Cfg::kTileN + static_cast<int>(rank) * Cfg::kBnCta;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % Cfg::kStages;
          const uint32_t ph = (it / Cfg::kStages) & 1;
          if (!dev::mbar_wait_bounded(dev::smem_addr(&empty[s]), ph ^ 1) ||
              *(volatile int *)&abort_flag) {
            dev::report_status(status, CMB_ERR_TIMEOUT);
            atomicExch(&abort_flag, 1);
            ok = false;
            break;
          }
          uint8_t *a_dst = ring + (size_t)s * Cfg::kStageBytes;
          uint8_t *b_dst = a_dst + Cfg::kABytes;
          const int kx = kb * Cfg::kBk;
          const uint32_t bar = dev::smem_addr(&full[s]);
          // B sub-tile u covers output columns [u * 256, u * 256 + 256) of the
          // tile; this CTA loads its kBnCta rows of each.
          if constexpr (CG == 1) {
            dev::mbar_arrive_expect_tx(bar, Cfg::kStageBytes);
            dev::tma_load_2d(dev::smem_addr(a_dst), &tmA, kx, a_row, bar);
#pragma unroll
            for (int u = 0; u < NSUB; ++u)
              dev::tma_load_2d(dev::smem_addr(b_dst + u * Cfg::kBSubBytes), &tmB, kx,
                               b_row + u * Cfg::kBn, bar);
          } else {
            const uint32_t leader_bar = tc::map_to_cta(bar, 0);
            if (rank == 0) dev::mbar_arrive_expect_tx(bar, 2 * Cfg::kStageBytes);
            tc::tma_load_2d_pair(dev::smem_addr(a_dst), &tmA, kx, a_row, leader_bar);
#pragma unroll
            for (int u = 0; u < NSUB; ++u)
              tc::tma_load_2d_pair(dev::smem_addr(b_dst + u * Cfg::kBSubBytes), &tmB, kx,
                                   b_row + u * Cfg::kBn, leader_bar);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0 && Cfg::kHeld) {
      // ------------------------------------------- MMA issuer, held epilogue
      // The two N=256 halves of the accumulator come back from the epilogue
      // one after the other.  Each tile starts with the MMAs of half 0 over
      // every stage already in the ring, then waits for half 1, issues its
      // MMAs over the same stages and frees them; the rest of K runs both
      // halves per stage.  Each half still accumulates in K order.
      int it = 0, j = 0;
      bool ok = true;
      const int pre = kblocks < Cfg::kStages ? kblocks : Cfg::kStages;
      for (int t = t_first; t < t_end && ok; t += t_step, ++j) {
        const uint32_t aph = static_cast<uint32_t>(j) & 1;
        for (int u = 0; u < 2 && ok; ++u) {
          if (!dev::mbar_wait_bounded(dev::smem_addr(&tempty[u]), aph ^ 1) ||
              *(volatile int *)&abort_flag) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          for (int kb = 0; kb < pre; ++kb) {
            const int s = (it + kb) % Cfg::kStages;
            const uint32_t ph = ((it + kb) / Cfg::kStages) & 1;
            if (u == 0) {
              if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), ph) ||
                  *(volatile int *)&abort_flag) {
                ok = false;
                break;
              }
              tc::fence_after_sync();
            }
            const uint32_t a_addr = dev::smem_addr(ring + (size_t)s * Cfg::kStageBytes);
            const uint64_t da = tc::sw128_kmajor_desc(a_addr);
            const uint64_t db = tc::sw128_kmajor_desc(a_addr + Cfg::kABytes);
#pragma unroll
            for (int k = 0; k < Cfg::kMmaPerStage; ++k)
              tc::mma<CG, kFp8>(tmem_base + u * Cfg::kBn, da + 2 * k,
                                db + (u * Cfg::kBSubBytes >> 4) + 2 * k, Cfg::kIdesc,
                                (kb | k) != 0 ? 1u : 0u);
            if (u == 1) {
              const uint32_t eb = dev::smem_addr(&empty[s]);
              tc::commit<CG>(eb);
              if constexpr (CG == 2) tc::commit<CG>(tc::map_to_cta(eb, 1));
            }
          }
        }
        if (!ok) break;
        it += pre;
        for (int kb = pre; kb < kblocks; ++kb, ++it) {
          const int s = it % Cfg::kStages;
          const uint32_t ph = (it / Cfg::kStages) & 1;
          if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), ph) ||
              *(volatile int *)&abort_flag) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t a_addr = dev::smem_addr(ring + (size_t)s * Cfg::kStageBytes);
          const uint64_t da = tc::sw128_kmajor_desc(a_addr);
          const uint64_t db = tc::sw128_kmajor_desc(a_addr + Cfg::kABytes);
#pragma unroll
          for (int k = 0; k < Cfg::kMmaPerStage; ++k)
#pragma unroll
            for (int u = 0; u < 2; ++u)
              tc::mma<CG, kFp8>(tmem_base + u * Cfg::kBn, da + 2 * k,
                                db + (u * Cfg::kBSubBytes >> 4) + 2 * k, Cfg::kIdesc, 1u);
          const uint32_t eb = dev::smem_addr(&empty[s]);
          tc::commit<CG>(eb);
          if constexpr (CG == 2) tc::commit<CG>(tc::map_to_cta(eb, 1));
        }
        if (!ok) break;
        const uint32_t fb = dev::smem_addr(&tfull[0]);
        tc::commit<CG>(fb);
        if constexpr (CG == 2) tc::commit<CG>(tc::map_to_cta(fb, 1));
      }
      if (!ok) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        atomicExch(&abort_flag, 1);
      }
      tc::commit<CG>(dev::smem_addr(&mma_done));
      if (!dev::mbar_wait_bounded(dev::smem_addr(&mma_done), 0))
        dev::report_status(status, CMB_ERR_TIMEOUT);
    } else if (lane == 0 && rank == 0) {
      // --------------------------------------------------------- MMA issuer
      int it = 0, j = 0;
      bool ok = true;
      for (int t = t_first; t < t_end && ok; t += t_step, ++j) {
        const int a = j % Cfg::kAccBufs;
        const uint32_t aph = (j / Cfg::kAccBufs) & 1;
        if (!dev::mbar_wait_bounded(dev::smem_addr(&tempty[a]), aph ^ 1)) {
          dev::report_status(status, CMB_ERR_TIMEOUT);
          atomicExch(&abort_flag, 1);
          break;
        }
        tc::fence_after_sync();
        const uint32_t d = tmem_base + static_cast<uint32_t>(a * Cfg::kTileN);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % Cfg::kStages;
          const uint32_t ph = (it / Cfg::kStages) & 1;
          if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), ph) ||
              *(volatile int *)&abort_flag) {
            dev::report_status(status, CMB_ERR_TIMEOUT);
            atomicExch(&abort_flag, 1);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t a_addr = dev::smem_addr(ring + (size_t)s * Cfg::kStageBytes);
          const uint64_t da = tc::sw128_kmajor_desc(a_addr);
          const uint64_t db = tc::sw128_kmajor_desc(a_addr + Cfg::kABytes);
#pragma unroll
          for (int k = 0; k < Cfg::kMmaPerStage; ++k)
#pragma unroll
            for (int u = 0; u < NSUB; ++u)
              tc::mma<CG, kFp8>(d + u * Cfg::kBn, da + 2 * k,
                                db + (u * Cfg::kBSubBytes >> 4) + 2 * k, Cfg::kIdesc,
                                (kb | k) != 0 ? 1u : 0u);
          const uint32_t eb = dev::smem_addr(&empty[s]);
          tc::commit<CG>(eb);
          if constexpr (CG == 2) tc::commit<CG>(tc::map_to_cta(eb, 1));
        }
        if (!ok) break;
        const uint32_t fb = dev::smem_addr(&tfull[a]);
        tc::commit<CG>(fb);
        if constexpr (CG == 2) tc::commit<CG>(tc::map_to_cta(fb, 1));
      }
      // All MMAs this thread issued have completed once mma_done flips.
      tc::commit<CG>(dev::smem_addr(&mma_done));
      if (!dev::mbar_wait_bounded(dev::smem_addr(&mma_done), 0))
        dev::report_status(status, CMB_ERR_TIMEOUT);
    }
  } else if constexpr (Cfg::kHeld) {
    // ---------------------------------------------------- held epilogue
    // Warp w reads TMEM lane quarter w % 4; the two warps of a quarter take
    // 128 columns each of one N=256 half.  Per half: four 32-column TMEM
    // loads into registers, hand the half back to the MMA issuer, then write
    // four 32 x 32 boxes (TMA store through the warp's staging box, or
    // streaming stores).
    const int q = warp & 3;
    const int ew = warp - 2;
    const int h = ew >> 2;
    float scale = 1.0f;
    if constexpr (kFp8) scale = __ldg(scale_a) * __ldg(scale_b);
    const bool vec_ok = (N % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    uint8_t *box = ring + (size_t)Cfg::kStages * Cfg::kStageBytes + (size_t)ew * Cfg::kEpiBoxBytes;
    uint32_t epi_count = 0;
    int j = 0;
    for (int t = t_first; t < t_end; t += t_step, ++j) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, group_m, tm, tn);
      if (!dev::mbar_wait_bounded(dev::smem_addr(&tfull[0]), static_cast<uint32_t>(j) & 1) ||
          *(volatile int *)&abort_flag) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        atomicExch(&abort_flag, 1);
        break;
      }
      tc::fence_after_sync();
      const int row0 = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kBmCta + q * 32;
      const int row = row0 + lane;
      float *crow = C + (size_t)row * N;
#pragma unroll 1
      for (int u = 0; u < 2; ++u) {
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               static_cast<uint32_t>(u * Cfg::kBn + h * 128);
        uint32_t r[4][32];
#pragma unroll
        for (int i = 0; i < 4; ++i) tc::ld_32x32b_x32(taddr + 32 * i, r[i]);
        tc::wait_ld();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          const uint32_t eb = dev::smem_addr(&tempty[u]);
          if constexpr (CG == 1) dev::mbar_arrive(eb);
          else dev::mbar_arrive_cluster(tc::map_to_cta(eb, 0));
        }
        if constexpr (kBf16Out) {
          // bf16 C: two 32 x 64 boxes (128-byte rows) per half, staged with
          // the same 128-byte swizzle; 16-byte piece p of a row holds
          // columns 8p .. 8p+7.
#pragma unroll
          for (int i2 = 0; i2 < 2; ++i2) {
            const int col0 = tn * Cfg::kTileN + u * Cfg::kBn + h * 128 + 64 * i2;
            uint32_t w[8][4];
#pragma unroll
            for (int p = 0; p < 8; ++p)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int ci = 2 * i2 + (p >> 2), c = (p & 3) * 8 + 2 * e;
                w[p][e] = pack_bf16x2(scale * __uint_as_float(r[ci][c]),
                                      scale * __uint_as_float(r[ci][c + 1]));
              }
            if constexpr (kTmaEpi) {
              if (row0 < M && col0 < N) {  // warp-uniform
                if (epi_count != 0) {
                  if (lane == 0) dev::bulk_wait_group_read<0>();
                  __syncwarp();
                }
                const uint32_t rb = dev::smem_addr(box) + lane * 128;
#pragma unroll
                for (int p = 0; p < 8; ++p) {
                  const uint32_t addr = rb + ((static_cast<uint32_t>(p) ^ (lane & 7)) << 4);
                  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w[p][0]),
                               "r"(w[p][1]), "r"(w[p][2]), "r"(w[p][3])
                               : "memory");
                }
                dev::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  dev::tma_store_2d(&tmC, col0, row0, dev::smem_addr(box));
                  dev::bulk_commit_group();
                }
                ++epi_count;
              }
            } else if (row < M) {
              __nv_bfloat16 *brow = Cb + (size_t)row * N;
              if (vec_ok && (N % 8 == 0) && col0 + 64 <= N) {
#pragma unroll
                for (int p = 0; p < 8; ++p)
                  st_cs_u4(brow + col0 + 8 * p, w[p][0], w[p][1], w[p][2], w[p][3]);
              } else {
#pragma unroll
                for (int p = 0; p < 8; ++p)
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const int c = col0 + 8 * p + 2 * e;
                    const uint32_t v = w[p][e];
                    if (c < N) brow[c] = __ushort_as_bfloat16(static_cast<unsigned short>(v));
                    if (c + 1 < N) brow[c + 1] = __ushort_as_bfloat16(static_cast<unsigned short>(v >> 16));
                  }
              }
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int col0 = tn * Cfg::kTileN + u * Cfg::kBn + h * 128 + 32 * i;
            if constexpr (kTmaEpi) {
              // Same 128-byte-swizzled staging as the two-box epilogue; the
              // one box is rewritten only after the store that last read it.
              if (row0 < M && col0 < N) {  // warp-uniform
                if (epi_count != 0) {
                  if (lane == 0) dev::bulk_wait_group_read<0>();
                  __syncwarp();
                }
                const uint32_t rb = dev::smem_addr(box) + lane * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                  const uint32_t addr = rb + ((static_cast<uint32_t>(c) ^ (lane & 7)) << 4);
                  asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr),
                               "f"(scale * __uint_as_float(r[i][4 * c])),
                               "f"(scale * __uint_as_float(r[i][4 * c + 1])),
                               "f"(scale * __uint_as_float(r[i][4 * c + 2])),
                               "f"(scale * __uint_as_float(r[i][4 * c + 3]))
                               : "memory");
                }
                dev::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  dev::tma_store_2d(&tmC, col0, row0, dev::smem_addr(box));
                  dev::bulk_commit_group();
                }
                ++epi_count;
              }
            } else if (row < M) {
              if (vec_ok && col0 + 32 <= N) {
#pragma unroll
                for (int c = 0; c < 32; c += 4)
                  st_cs_f4(crow + col0 + c, scale * __uint_as_float(r[i][c]),
                           scale * __uint_as_float(r[i][c + 1]), scale * __uint_as_float(r[i][c + 2]),
                           scale * __uint_as_float(r[i][c + 3]));
              } else {
#pragma unroll
                for (int c = 0; c < 32; ++c)
                  if (col0 + c < N) crow[col0 + c] = scale * __uint_as_float(r[i][c]);
              }
            }
          }
        }
      }
    }
    if constexpr (kTmaEpi) {
      if (lane == 0) dev::bulk_wait_group<0>();  // stores complete before the CTA leaves
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w reads TMEM lane quarter w % 4; with 8 epilogue warps two warps
    // share a quarter and split its columns in halves.
    const int q = warp & 3;
    const int ew = warp - 2;
    constexpr int kChunks = Cfg::kTileN / 32 / (EPIW / 4);  // 32-column chunks per warp
    const int c_begin = (ew / 4) * kChunks;
    float scale = 1.0f;
    if constexpr (kFp8) scale = __ldg(scale_a) * __ldg(scale_b);
    const bool vec_ok = (N % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
    uint8_t *epi = ring + (size_t)Cfg::kStages * Cfg::kStageBytes + (size_t)ew * 2 * Cfg::kEpiBoxBytes;
    uint32_t epi_count = 0;
    int j = 0;
    for (int t = t_first; t < t_end; t += t_step, ++j) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, group_m, tm, tn);
      const int a = j % Cfg::kAccBufs;
      const uint32_t ph = (j / Cfg::kAccBufs) & 1;
      if (!dev::mbar_wait_bounded(dev::smem_addr(&tfull[a]), ph) ||
          *(volatile int *)&abort_flag) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        atomicExch(&abort_flag, 1);
        break;
      }
      tc::fence_after_sync();
      const int row0 = tm * Cfg::kTileM + static_cast<int>(rank) * Cfg::kBmCta + q * 32;
      const int row = row0 + lane;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(a * Cfg::kTileN);
      float *crow = C + (size_t)row * N;
#pragma unroll 1
      for (int c = c_begin; c < c_begin + kChunks; ++c) {
        uint32_t r[32];
        tc::ld_32x32b_x32(taddr + c * 32, r);
        tc::wait_ld();
        if (c == c_begin + kChunks - 1) {
          // every TMEM read of this accumulator is done: hand it back
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) {
            const uint32_t eb = dev::smem_addr(&tempty[a]);
            if constexpr (CG == 1) dev::mbar_arrive(eb);
            else dev::mbar_arrive_cluster(tc::map_to_cta(eb, 0));
          }
        }
        const int col0 = tn * Cfg::kTileN + c * 32;
        if constexpr (kTmaEpi) {
          // Stage the warp's 32 x 32 box in shared memory (128-byte
          // swizzle: 16-byte chunk j of row r at (j ^ (r % 8)) * 16, which
          // also keeps the 8 lanes of each store phase on distinct banks)
          // and write it out with one tiled TMA store.  Boxes wholly outside
          // C are skipped without touching a buffer, so every buffer reuse
          // follows the committed store that last read it.
          if (row0 < M && col0 < N) {  // warp-uniform
            uint8_t *box = epi + (size_t)(epi_count & 1) * Cfg::kEpiBoxBytes;
            if (lane == 0) dev::bulk_wait_group_read<1>();  // the store 2 boxes ago has read it
            __syncwarp();
            const uint32_t rb = dev::smem_addr(box) + lane * 128;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t addr = rb + ((static_cast<uint32_t>(j) ^ (lane & 7)) << 4);
              asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr),
                           "f"(scale * __uint_as_float(r[4 * j])),
                           "f"(scale * __uint_as_float(r[4 * j + 1])),
                           "f"(scale * __uint_as_float(r[4 * j + 2])),
                           "f"(scale * __uint_as_float(r[4 * j + 3]))
                           : "memory");
            }
            dev::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              dev::tma_store_2d(&tmC, col0, row0, dev::smem_addr(box));
              dev::bulk_commit_group();
            }
            ++epi_count;
          }
        } else if (row < M) {
          if (vec_ok && col0 + 32 <= N) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              st_cs_f4(crow + col0 + i, scale * __uint_as_float(r[i]),
                       scale * __uint_as_float(r[i + 1]), scale * __uint_as_float(r[i + 2]),
                       scale * __uint_as_float(r[i + 3]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < N) crow[col0 + i] = scale * __uint_as_float(r[i]);
          }
        }
      }
    }
    if constexpr (kTmaEpi) {
      if (lane == 0) dev::bulk_wait_group<0>();  // stores complete before the CTA leaves
      __syncwarp();
    }
  }

  // ------------------------------------------------------------- teardown
  tc::fence_before_sync();
  __syncthreads();
  if constexpr (CG == 2) tc::cluster_sync();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc<CG>(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------ e4m3 quantisation

__global__ void k_amax_bf16(const __nv_bfloat16 *__restrict__ x, size_t n, float *amax) {
  float m = 0.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  // non-negative floats order like their bit patterns
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int *>(amax), __float_as_uint(m));
}

// q = e4m3_satfinite(x * (448 / amax)); scale_out[0] = amax / 448 (the
// factor that turns q back into x).
__global__ void k_quantize_e4m3(const __nv_bfloat16 *__restrict__ x, size_t n,
                                __nv_fp8_storage_t *__restrict__ q, float *scale_out) {
  const float amax = scale_out[1];
  const float inv = amax > 0.0f ? __fdiv_rn(448.0f, amax) : 1.0f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    q[i] = __nv_cvt_float_to_fp8(__fmul_rn(__bfloat162float(x[i]), inv), __NV_SATFINITE,
                                 __NV_E4M3);
  if (blockIdx.x == 0 && threadIdx.x == 0)
    scale_out[0] = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
}

// Installed die maps, per device: SMs on each die (0 / 0 = none installed).
constexpr int kMaxDevices = 64;
std::mutex g_die_mu;
int g_die_sms[kMaxDevices][2];
std::atomic<unsigned> g_claim_seq{0};

// Clusters that work in die 0's tile range (the rest work in die 1's), or
// -1 for the plain order when no map is installed on the current device;
// `slot` = the claim counters this launch uses.
void die_split(int cg, int clusters, int *pairs0, int *slot) {
  *pairs0 = -1;
  *slot = 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  int sms[2];
  {
    std::lock_guard<std::mutex> lk(g_die_mu);
    sms[0] = g_die_sms[dev][0];
    sms[1] = g_die_sms[dev][1];
  }
  const int cap0 = sms[0] / cg, cap1 = sms[1] / cg;
  if (cap0 + cap1 <= 0) return;
  long p0 = std::lround(static_cast<double>(clusters) * cap0 / (cap0 + cap1));
  if (p0 < 0) p0 = 0;
  if (p0 > clusters) p0 = clusters;
  *pairs0 = static_cast<int>(p0);
  *slot = static_cast<int>(g_claim_seq.fetch_add(1u, std::memory_order_relaxed) % kClaimSlots);
}

template <int CG, bool kFp8, int STAGES, bool kTmaEpi, int NSUB, int EPIW, bool kBf16Out = false>
int launch_gemm(const void *A, const void *B, void *C, int M, int N, int K,
                const float *scale_a, const float *scale_b, int group_m, int *status,
                cudaStream_t stream) {
  using Cfg = GemmCfg<CG, kFp8, STAGES, kTmaEpi, NSUB, EPIW>;
  const CUtensorMapDataType dt =
      kFp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, dt, A, M, K, (uint64_t)K * Cfg::kElem, Cfg::kBmCta, Cfg::kBk,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, dt, B, N, K, (uint64_t)K * Cfg::kElem, Cfg::kBnCta, Cfg::kBk,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  CUtensorMap tcm;
  if constexpr (kTmaEpi && kBf16Out) {
    rc = make_tmap_2d(&tcm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, M, N, (uint64_t)N * 2, 32, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (rc) return rc;
  } else if constexpr (kTmaEpi) {
    rc = make_tmap_2d(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, M, N, (uint64_t)N * 4, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (rc) return rc;
  } else {
    tcm = ta;  // unused
  }
  auto kern = k_gemm<CG, kFp8, STAGES, kTmaEpi, NSUB, EPIW, kBf16Out>;
  CMB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(Cfg::kSmem)));
  const int tiles = ((M + Cfg::kTileM - 1) / Cfg::kTileM) * ((N + Cfg::kTileN - 1) / Cfg::kTileN);
  int clusters = current_sm_count() / CG;
  if (clusters > tiles) clusters = tiles;
  if (group_m <= 0) group_m = 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * CG));
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int die_pairs0, claim_slot;
  die_split(CG, clusters, &die_pairs0, &claim_slot);
  CMB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tb, tcm, C, M, N, K, scale_a, scale_b,
                                  group_m, die_pairs0, claim_slot, status));
  return CMB_OK;
}

int gemm_checks(const char *fn, const void *A, const void *B, const float *C, int M, int N, int K,
                int elem, int cta_group) {
  if (A == nullptr || B == nullptr || C == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "%s: null operand", fn);
  if (M <= 0 || N <= 0 || K <= 0) return fail(CMB_ERR_INVALID_ARG, "%s: empty GEMM", fn);
  if ((static_cast<long long>(K) * elem) % 16 != 0)
    return fail(CMB_ERR_INVALID_ARG, "%s: K*%d bytes must be a multiple of 16", fn, elem);
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    return fail(CMB_ERR_INVALID_ARG, "%s: A and B must be 16-byte aligned", fn);
  if (cta_group != 1 && cta_group != 2)
    return fail(CMB_ERR_INVALID_ARG, "%s: cta_group %d not 1 or 2", fn, cta_group);
  if (current_cc() != 100)
    return fail(CMB_ERR_UNSUPPORTED, "%s: needs an sm_100 device (found cc %d)", fn, current_cc());
  return CMB_OK;
}

// Default shapes (from sweeps on B200 against cuBLAS measured alongside):
// 1-CTA 128x256 tiles with 4 stages of 48 KiB and 4 epilogue warps; 2-CTA
// 256x512 tiles with 4 stages of 48 KiB per CTA and the 8-warp held
// epilogue (1-3 % over 4 warps: the MMAs of the next tile restart after
// half of the drain); raster groups of 8 tile rows; the TMA-store epilogue
// whenever C's row pitch allows a tensor map (N % 4 == 0, 16-byte aligned
// C).
template <bool kFp8, bool kTmaEpi>
int dispatch_stages(const void *A, const void *B, float *C, int M, int N, int K,
                    const float *scale_a, const float *scale_b, int cta_group, int stages,
                    int group_m, int tile_n, int epi_warps, int *status, cudaStream_t stream) {
#define CMB_GEMM_CASE(CGV, S, NS, EW)                                                          \
  if (cta_group == CGV && stages == S && tile_n == 256 * NS && epi_warps == EW)               \
    return launch_gemm<CGV, kFp8, S, kTmaEpi, NS, EW>(A, B, C, M, N, K, scale_a, scale_b,      \
                                                      group_m, status, stream);
  if (tile_n == 0) tile_n = cta_group == 2 ? 512 : 256;
  if (stages == 0) stages = 4;
  if (epi_warps == 0) epi_warps = tile_n == 512 ? 8 : 4;
  CMB_GEMM_CASE(1, 3, 1, 4)
  CMB_GEMM_CASE(1, 4, 1, 4)
  CMB_GEMM_CASE(2, 4, 1, 4)
  CMB_GEMM_CASE(2, 5, 1, 4)
  CMB_GEMM_CASE(2, 6, 1, 4)
  CMB_GEMM_CASE(2, 3, 2, 4)
  CMB_GEMM_CASE(2, 4, 2, 4)
  CMB_GEMM_CASE(2, 3, 2, 8)
  CMB_GEMM_CASE(2, 4, 2, 8)
  if constexpr (!kTmaEpi) {
    CMB_GEMM_CASE(2, 7, 1, 4)
  }
#undef CMB_GEMM_CASE
  return fail(CMB_ERR_INVALID_ARG,
              "gemm: no kernel for cta_group %d, %d stages, tile_n %d, %d epilogue warps",
              cta_group, stages, tile_n, epi_warps);
}

template <bool kFp8>
int dispatch_gemm(const void *A, const void *B, float *C, int M, int N, int K,
                  const float *scale_a, const float *scale_b, int cta_group, int stages,
                  int group_m, int epilogue, int tile_n, int epi_warps, int *status,
                  cudaStream_t stream) {
  const bool tma_ok = (N % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
  if (epilogue == 0) epilogue = tma_ok ? 2 : 1;
  if (epilogue == 2 && !tma_ok)
    return fail(CMB_ERR_INVALID_ARG, "gemm: the TMA-store epilogue needs N %% 4 == 0 and a "
                "16-byte aligned C");
  if (epilogue == 2)
    return dispatch_stages<kFp8, true>(A, B, C, M, N, K, scale_a, scale_b, cta_group, stages,
                                       group_m, tile_n, epi_warps, status, stream);
  if (epilogue == 1)
    return dispatch_stages<kFp8, false>(A, B, C, M, N, K, scale_a, scale_b, cta_group, stages,
                                        group_m, tile_n, epi_warps, status, stream);
  return fail(CMB_ERR_INVALID_ARG, "gemm: epilogue %d not in {0, 1, 2}", epilogue);
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_gemm_bf16(const void *A, const void *B, float *C, int M, int N, int K,
                             int cta_group, int *status, cmb_stream_t stream) {
  int rc = gemm_checks("cmb_gemm_bf16", A, B, C, M, N, K, 2, cta_group);
  if (rc) return rc;
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  return dispatch_gemm<false>(A, B, C, M, N, K, nullptr, nullptr, cta_group, 0, 0, 0, 0, 0,
                              status, stream);
}

extern "C" int cmb_gemm_tuned(const void *A, const void *B, float *C, int M, int N, int K,
                              int fp8, const float *scale_a, const float *scale_b, int cta_group,
                              int stages, int group_m, int epilogue, int tile_n, int epi_warps,
                              int *status, cmb_stream_t stream) {
  int rc = gemm_checks("cmb_gemm_tuned", A, B, C, M, N, K, fp8 ? 1 : 2, cta_group);
  if (rc) return rc;
  if (fp8 && (scale_a == nullptr || scale_b == nullptr))
    return fail(CMB_ERR_INVALID_ARG, "cmb_gemm_tuned: null scale");
  if (group_m < 0) return fail(CMB_ERR_INVALID_ARG, "cmb_gemm_tuned: group_m < 0");
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  return fp8 ? dispatch_gemm<true>(A, B, C, M, N, K, scale_a, scale_b, cta_group, stages, group_m,
                                   epilogue, tile_n, epi_warps, status, stream)
             : dispatch_gemm<false>(A, B, C, M, N, K, nullptr, nullptr, cta_group, stages,
                                    group_m, epilogue, tile_n, epi_warps, status, stream);
}

extern "C" int cmb_gemm_e4m3(const void *A, const void *B, float *C, int M, int N, int K,
                             const float *scale_a, const float *scale_b, int cta_group,
                             int *status, cmb_stream_t stream) {
  int rc = gemm_checks("cmb_gemm_e4m3", A, B, C, M, N, K, 1, cta_group);
  if (rc) return rc;
  if (scale_a == nullptr || scale_b == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_gemm_e4m3: null scale");
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  return dispatch_gemm<true>(A, B, C, M, N, K, scale_a, scale_b, cta_group, 0, 0, 0, 0, 0,
                             status, stream);
}

extern "C" int cmb_gemm_bf16_out(const void *A, const void *B, void *C, int M, int N, int K,
                                 int fp8, const float *scale_a, const float *scale_b, int *status,
                                 cmb_stream_t stream) {
  int rc = gemm_checks("cmb_gemm_bf16_out", A, B, static_cast<const float *>(C), M, N, K,
                       fp8 ? 1 : 2, 2);
  if (rc) return rc;
  if (fp8 && (scale_a == nullptr || scale_b == nullptr))
    return fail(CMB_ERR_INVALID_ARG, "cmb_gemm_bf16_out: null scale");
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  // the TMA-store epilogue when C's row pitch allows a tensor map
  const bool tma_ok = (N % 8 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15) == 0);
  if (fp8)
    return tma_ok ? launch_gemm<2, true, 4, true, 2, 8, true>(A, B, C, M, N, K, scale_a, scale_b, 8,
                                                              status, stream)
                  : launch_gemm<2, true, 4, false, 2, 8, true>(A, B, C, M, N, K, scale_a, scale_b,
                                                               8, status, stream);
  return tma_ok ? launch_gemm<2, false, 4, true, 2, 8, true>(A, B, C, M, N, K, nullptr, nullptr, 8,
                                                             status, stream)
                : launch_gemm<2, false, 4, false, 2, 8, true>(A, B, C, M, N, K, nullptr, nullptr, 8,
                                                              status, stream);
}

namespace cmb {
void gemm_release_die_map(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lk(g_die_mu);
  g_die_sms[dev][0] = g_die_sms[dev][1] = 0;
}
}  // namespace cmb

extern "C" int cmb_gemm_set_sm_die_map(const uint8_t *sm_die, int n_ids) {
  int count[2] = {0, 0};
  uint8_t map[CMB_DIE_MAP_IDS] = {0};
  const bool clear = sm_die == nullptr || n_ids == 0;
  if (!clear) {
    if (n_ids < 0 || n_ids > CMB_DIE_MAP_IDS)
      return fail(CMB_ERR_INVALID_ARG, "cmb_gemm_set_sm_die_map: %d ids, not 1-%d", n_ids,
                  CMB_DIE_MAP_IDS);
    for (int i = 0; i < n_ids; ++i) {
      if (sm_die[i] == 0xFF) continue;  // no SM with this id
      if (sm_die[i] > 1)
        return fail(CMB_ERR_INVALID_ARG, "cmb_gemm_set_sm_die_map: SM %d on die %d, not 0 or 1",
                    i, sm_die[i]);
      map[i] = sm_die[i];
      ++count[sm_die[i]];
    }
    if (count[0] == 0 || count[1] == 0)
      return fail(CMB_ERR_INVALID_ARG,
                  "cmb_gemm_set_sm_die_map: both dies need SMs (%d / %d)", count[0], count[1]);
  }
  int dev = -1;
  CMB_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(CMB_ERR_UNSUPPORTED, "cmb_gemm_set_sm_die_map: device %d", dev);
  if (!clear) CMB_CUDA_TRY(cudaMemcpyToSymbol(g_sm_die, map, sizeof(map)));
  std::lock_guard<std::mutex> lk(g_die_mu);
  g_die_sms[dev][0] = count[0];
  g_die_sms[dev][1] = count[1];
  return CMB_OK;
}

extern "C" int cmb_quantize_e4m3(const uint16_t *src_bf16, size_t n, uint8_t *dst,
                                 float *scale_out, cmb_stream_t stream) {
  if (src_bf16 == nullptr || dst == nullptr || scale_out == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_quantize_e4m3: null pointer");
  CMB_CUDA_TRY(cudaMemsetAsync(scale_out, 0, 2 * sizeof(float), stream));
  if (n == 0) return CMB_OK;
  size_t grid = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(current_sm_count()) * 8;
  if (grid > cap) grid = cap;
  const auto *x = reinterpret_cast<const __nv_bfloat16 *>(src_bf16);
  k_amax_bf16<<<static_cast<int>(grid), 256, 0, stream>>>(x, n, scale_out + 1);
  CMB_LAUNCH_CHECK();
  k_quantize_e4m3<<<static_cast<int>(grid), 256, 0, stream>>>(
      x, n, reinterpret_cast<__nv_fp8_storage_t *>(dst), scale_out);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
