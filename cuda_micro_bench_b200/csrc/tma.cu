// tma.cu — TMA bulk-tensor probes (reference src/tma.cu).
//
// k_tma_tile_copy: a 2-D bf16 matrix moved tile by tile with
// cp.async.bulk.tensor: one thread (warp 0) loads box_rows x box_cols tiles
// into a STAGES-deep shared-memory ring, each completion counted on the
// stage's full mbarrier (expect_tx); a second thread (warp 1) stores each
// tile back out with a tiled TMA store from the same buffer and hands the
// stage back (empty mbarrier) once the store has finished reading it; up to
// STAGES / 2 stores read the ring at once.
// Persistent grid: CTAs stride over the tile list.  In load-only mode (the
// reference's G2S bandwidth probe, src/tma.cu:72-121) the second thread
// only folds the first 16 bytes of each tile into a per-CTA XOR so the
// loads stay observable.
//
// k_tma_1d_latency: one thread issues a 16-byte 1-D TMA load and waits for
// it, `iters` times (src/tma.cu:20-69).
//
// Every wait is bounded (cmb_device.cuh); no load names a destination in
// another CTA or another GPU.
#include <cuda.h>

#include <mutex>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major tensor map: dims {cols, rows}, row pitch in bytes.
int make_tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t rows,
                 uint64_t cols, uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols,
                 CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return fail(CMB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(CMB_ERR_INVALID_ARG, "cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u",
                static_cast<int>(r), (unsigned long long)rows, (unsigned long long)cols, box_rows,
                box_cols);
  return CMB_OK;
}

namespace {

constexpr int kTmaThreads = 64;  // warp 0: loads, warp 1: stores

struct TileShape {
  int rows, cols, box_rows, box_cols, tiles_x, tiles;
  int contiguous;  // 0: CTA b takes tiles b, b + grid, ...; 1: a contiguous run
  int evict_first;  // 1: loads and stores carry an L2 evict-first policy
};

// k-th tile of this CTA and the number of tiles it owns.
__device__ __forceinline__ int tile_of(const TileShape &s, int k) {
  if (s.contiguous) {
    const int per = (s.tiles + gridDim.x - 1) / gridDim.x;
    return blockIdx.x * per + k;
  }
  return blockIdx.x + k * gridDim.x;
}

__device__ __forceinline__ int tiles_of(const TileShape &s) {
  if (s.contiguous) {
    const int per = (s.tiles + gridDim.x - 1) / gridDim.x;
    const int first = blockIdx.x * per;
    return first >= s.tiles ? 0 : min(per, s.tiles - first);
  }
  return blockIdx.x < s.tiles ? (s.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
}

template <int STAGES, bool kStore>
__global__ void __launch_bounds__(kTmaThreads, 1)
    k_tma_tile_copy(const __grid_constant__ CUtensorMap src_map,
                    const __grid_constant__ CUtensorMap dst_map, TileShape shape,
                    uint32_t tile_bytes, int *status, uint32_t *xor_out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned ring (TMA needs 128-byte aligned destinations).
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES];
  __shared__ int abort_flag, loads_issued, tiles_consumed;

  // stores in flight per CTA: half the ring
  constexpr int kLag = STAGES / 2 > 1 ? STAGES / 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(dev::smem_addr(&full[s]), 1);
      dev::mbar_init(dev::smem_addr(&empty[s]), 1);
    }
    abort_flag = 0;
    loads_issued = 0;
    tiles_consumed = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&src_map);
    if (kStore) dev::tma_prefetch_desc(&dst_map);
  }
  __syncthreads();

  const int my_tiles = tiles_of(shape);

  if (warp == 0 && lane == 0) {
    // producer
    int k = 0;
    for (; k < my_tiles; ++k) {
      const int s = k % STAGES, use = k / STAGES;
      if (use > 0 && !dev::mbar_wait_bounded(dev::smem_addr(&empty[s]), (use - 1) & 1)) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        atomicExch(&abort_flag, 1);
        break;
      }
      if (*(volatile int *)&abort_flag) break;
      const int t = tile_of(shape, k);
      const int ty = t / shape.tiles_x, tx = t - ty * shape.tiles_x;
      const uint32_t bar = dev::smem_addr(&full[s]);
      dev::mbar_arrive_expect_tx(bar, tile_bytes);
      if (shape.evict_first)
        dev::tma_load_2d_hint(dev::smem_addr(ring + (size_t)s * tile_bytes), &src_map,
                              tx * shape.box_cols, ty * shape.box_rows, bar,
                              dev::policy_evict_first());
      else
        dev::tma_load_2d(dev::smem_addr(ring + (size_t)s * tile_bytes), &src_map,
                         tx * shape.box_cols, ty * shape.box_rows, bar);
    }
    loads_issued = k;
  } else if (warp == 1 && lane == 0) {
    // consumer: store (or fold) each tile, then hand its stage back
    uint32_t x = 0;
    int k = 0;
    for (; k < my_tiles; ++k) {
      const int s = k % STAGES, use = k / STAGES;
      if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), use & 1)) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        atomicExch(&abort_flag, 1);
        break;
      }
      uint8_t *buf = ring + (size_t)s * tile_bytes;
      if (kStore) {
        const int t = tile_of(shape, k);
        const int ty = t / shape.tiles_x, tx = t - ty * shape.tiles_x;
        if (shape.evict_first)
          dev::tma_store_2d_hint(&dst_map, tx * shape.box_cols, ty * shape.box_rows,
                                 dev::smem_addr(buf), dev::policy_evict_first());
        else
          dev::tma_store_2d(&dst_map, tx * shape.box_cols, ty * shape.box_rows,
                            dev::smem_addr(buf));
        dev::bulk_commit_group();
        // Keep kLag stores reading shared memory at once: once only kLag
        // are pending, the store of tile k - kLag has read its stage.
        dev::bulk_wait_group_read<kLag>();
        if (k >= kLag) dev::mbar_arrive(dev::smem_addr(&empty[(k - kLag) % STAGES]));
      } else {
        const uint4 v = *reinterpret_cast<const uint4 *>(buf);
        x ^= v.x ^ v.y ^ v.z ^ v.w;
        dev::mbar_arrive(dev::smem_addr(&empty[s]));
      }
    }
    if (kStore) {
      dev::bulk_wait_group<0>();  // all stores complete and visible
    } else if (xor_out != nullptr) {
      xor_out[blockIdx.x] = x;
    }
    tiles_consumed = k;
  }
  __syncthreads();
  // After a failed wait: wait (bounded) for loads still in flight into the
  // ring before the CTA's shared memory goes away.
  if (threadIdx.x == 0 && tiles_consumed < loads_issued) {
    for (int k = tiles_consumed; k < loads_issued; ++k) {
      const int s = k % STAGES;
      if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), (k / STAGES) & 1, 100000000ull))
        break;
    }
  }
}

// TMA loads with load/store-unit stores: warp 0 fills the ring as above;
// kLsuStoreWarps warps copy each tile from shared memory into registers
// (16-byte vectors, consecutive threads on consecutive vectors of a row),
// hand the stage back as soon as their shared-memory reads are done, then
// write the registers out with streaming 16-byte stores, clipped at the
// matrix edge.  The stage is free before the stores complete, unlike a TMA
// store, which holds it until the store has read it.
constexpr int kLsuStoreWarps = 4;
constexpr int kLsuThreads = 32 * (1 + kLsuStoreWarps);
constexpr int kLsuVecs = 16;  // vectors per thread per round (one 32 KiB tile)

template <int STAGES>
__global__ void __launch_bounds__(kLsuThreads)
    k_tma_tile_copy_lsu(const __grid_constant__ CUtensorMap src_map, TileShape shape,
                        uint32_t tile_bytes, char *__restrict__ dst, int *status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES];
  __shared__ int abort_flag, loads_issued, tiles_consumed;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      dev::mbar_init(dev::smem_addr(&full[s]), 1);
      dev::mbar_init(dev::smem_addr(&empty[s]), kLsuStoreWarps);
    }
    abort_flag = 0;
    loads_issued = 0;
    tiles_consumed = 0;
    dev::fence_mbar_init();
    dev::tma_prefetch_desc(&src_map);
  }
  __syncthreads();
  const int my_tiles = tiles_of(shape);

  if (warp == 0) {
    if (lane == 0) {
      int k = 0;
      for (; k < my_tiles; ++k) {
        const int s = k % STAGES, use = k / STAGES;
        if (use > 0 && !dev::mbar_wait_bounded(dev::smem_addr(&empty[s]), (use - 1) & 1)) {
          dev::report_status(status, CMB_ERR_TIMEOUT);
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*(volatile int *)&abort_flag) break;
        const int t = tile_of(shape, k);
        const int ty = t / shape.tiles_x, tx = t - ty * shape.tiles_x;
        const uint32_t bar = dev::smem_addr(&full[s]);
        dev::mbar_arrive_expect_tx(bar, tile_bytes);
        dev::tma_load_2d(dev::smem_addr(ring + (size_t)s * tile_bytes), &src_map,
                         tx * shape.box_cols, ty * shape.box_rows, bar);
      }
      loads_issued = k;
    }
  } else {
    const int t = threadIdx.x - 32;                // 0 .. 32 * kLsuStoreWarps - 1
    constexpr int kT = 32 * kLsuStoreWarps;
    const int vpr = shape.box_cols / 8;            // 16-byte vectors per tile row
    const int nvec = static_cast<int>(tile_bytes / 16);
    int k = 0;
    for (; k < my_tiles; ++k) {
      const int s = k % STAGES;
      if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), (k / STAGES) & 1) ||
          *(volatile int *)&abort_flag) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        atomicExch(&abort_flag, 1);
        break;
      }
      const int tile = tile_of(shape, k);
      const int ty = tile / shape.tiles_x, tx = tile - ty * shape.tiles_x;
      const int row0 = ty * shape.box_rows, col0 = tx * shape.box_cols;
      const uint4 *buf = reinterpret_cast<const uint4 *>(ring + (size_t)s * tile_bytes);
      for (int base = 0; base < nvec; base += kT * kLsuVecs) {
        uint4 v[kLsuVecs];
#pragma unroll
        for (int j = 0; j < kLsuVecs; ++j) {
          const int i = base + j * kT + t;
          if (i < nvec) v[j] = buf[i];
        }
        if (base + kT * kLsuVecs >= nvec) {
          // every read of this stage by this warp is done: hand it back
          __syncwarp();
          if (lane == 0) dev::mbar_arrive(dev::smem_addr(&empty[s]));
        }
#pragma unroll
        for (int j = 0; j < kLsuVecs; ++j) {
          const int i = base + j * kT + t;
          if (i >= nvec) continue;
          const int r = i / vpr, c = i - r * vpr;
          const int grow = row0 + r, gcol = col0 + c * 8;
          if (grow < shape.rows && gcol < shape.cols)
            dev::st_stream_v4(dst + ((size_t)grow * shape.cols + gcol) * 2, v[j]);
        }
      }
    }
    if (t == 0) tiles_consumed = k;
  }
  __syncthreads();
  // After a failed wait: wait (bounded) for loads still in flight into the
  // ring before the CTA's shared memory goes away.
  if (threadIdx.x == 0 && tiles_consumed < loads_issued) {
    for (int k = tiles_consumed; k < loads_issued; ++k) {
      const int s = k % STAGES;
      if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), (k / STAGES) & 1, 100000000ull))
        break;
    }
  }
}

__global__ void k_tma_1d_latency(const __grid_constant__ CUtensorMap map, int x, int iters,
                                 uint32_t *out_cycles, uint8_t *landed, int *status) {
  __shared__ __align__(128) uint8_t buf[128];
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = dev::smem_addr(&bar);
  dev::mbar_init(b, 1);
  dev::fence_mbar_init();
  // The destination starts zeroed, so the bytes read back after the loop
  // can only have come from the loads.
  reinterpret_cast<uint4 *>(buf)[0] = make_uint4(0u, 0u, 0u, 0u);
  dev::fence_proxy_async_smem();
  uint32_t done = 0;
  const uint64_t t0 = dev::clock64();
  for (int i = 0; i < iters; ++i) {
    dev::mbar_arrive_expect_tx(b, 16);
    dev::tma_load_1d(dev::smem_addr(buf), &map, x, b);
    if (!dev::mbar_wait_bounded(b, static_cast<uint32_t>(i & 1))) {
      dev::report_status(status, CMB_ERR_TIMEOUT);
      // the load may still land: wait once more before leaving
      dev::mbar_wait_bounded(b, static_cast<uint32_t>(i & 1), 100000000ull);
      return;
    }
    ++done;
  }
  const uint64_t t1 = dev::clock64_after(done + buf[0]);
  *out_cycles = static_cast<uint32_t>(t1 - t0);
  if (landed != nullptr) reinterpret_cast<uint4 *>(landed)[0] = reinterpret_cast<const uint4 *>(buf)[0];
}

template <int STAGES>
int launch_tile_lsu(const CUtensorMap &sm, TileShape shape, uint32_t tile_bytes, void *dst,
                    int *status, cudaStream_t stream, int grid) {
  const size_t smem = (size_t)STAGES * tile_bytes + 1024;
  auto kern = k_tma_tile_copy_lsu<STAGES>;
  CMB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  kern<<<grid, kLsuThreads, smem, stream>>>(sm, shape, tile_bytes, static_cast<char *>(dst),
                                            status);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

template <int STAGES, bool kStore>
int launch_tile(const CUtensorMap &sm, const CUtensorMap &dm, TileShape shape, uint32_t tile_bytes,
                int ctas_per_sm, int *status, uint32_t *xor_out, cudaStream_t stream, int grid) {
  const size_t smem = (size_t)STAGES * tile_bytes + 1024;
  auto kern = k_tma_tile_copy<STAGES, kStore>;
  CMB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  kern<<<grid, kTmaThreads, smem, stream>>>(sm, dm, shape, tile_bytes, status, xor_out);
  CMB_LAUNCH_CHECK();
  (void)ctas_per_sm;
  return CMB_OK;
}

int tile_impl(void *dst, const void *src, int rows, int cols, int box_rows, int box_cols,
              int stages, int ctas_per_sm, int *status, uint32_t *xor_out, int grid_override,
              int contiguous, cmb_stream_t stream) {
  const bool store = dst != nullptr;
  if (src == nullptr) return fail(CMB_ERR_INVALID_ARG, "tma tile: null src");
  if (rows <= 0 || cols <= 0) return fail(CMB_ERR_INVALID_ARG, "tma tile: empty matrix");
  if (cols % 8 != 0)
    return fail(CMB_ERR_INVALID_ARG, "tma tile: cols %d: the row pitch must be a multiple of 16 "
                "bytes", cols);
  if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return fail(CMB_ERR_INVALID_ARG, "tma tile: base addresses must be 16-byte aligned");
  if (box_rows < 1 || box_rows > 256 || box_cols < 8 || box_cols > 256 || box_cols % 8 != 0)
    return fail(CMB_ERR_INVALID_ARG, "tma tile: box %dx%d outside [1,256]x[8,256] (cols %% 8)",
                box_rows, box_cols);
  const uint32_t tile_bytes = static_cast<uint32_t>(box_rows) * box_cols * 2;
  if (tile_bytes % 1024 != 0)
    return fail(CMB_ERR_INVALID_ARG, "tma tile: box bytes %u not a multiple of 1024", tile_bytes);
  if (stages < 2 || stages > 8 || (size_t)stages * tile_bytes + 1024 > 227 * 1024)
    return fail(CMB_ERR_INVALID_ARG, "tma tile: %d stages of %u bytes exceed shared memory",
                stages, tile_bytes);
  if (ctas_per_sm < 1 || ctas_per_sm > 4)
    return fail(CMB_ERR_INVALID_ARG, "tma tile: ctas_per_sm %d not in [1,4]", ctas_per_sm);
  CUtensorMap sm, dm;
  int rc = make_tmap_2d(&sm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, src, rows, cols, (uint64_t)cols * 2,
                        box_rows, box_cols, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (rc) return rc;
  rc = make_tmap_2d(&dm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, store ? dst : src, rows, cols,
                    (uint64_t)cols * 2, box_rows, box_cols, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc) return rc;
  TileShape shape;
  shape.rows = rows;
  shape.cols = cols;
  shape.box_rows = box_rows;
  shape.box_cols = box_cols;
  shape.tiles_x = (cols + box_cols - 1) / box_cols;
  const long long tiles = (long long)shape.tiles_x * ((rows + box_rows - 1) / box_rows);
  if (tiles > 0x7fffffffLL) return fail(CMB_ERR_INVALID_ARG, "tma tile: too many tiles");
  shape.tiles = static_cast<int>(tiles);
  shape.contiguous = (contiguous & 1) ? 1 : 0;
  shape.evict_first = (contiguous & 2) ? 1 : 0;
  int grid = grid_override > 0 ? grid_override : current_sm_count() * ctas_per_sm;
  if (grid > shape.tiles) grid = shape.tiles;
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  const bool lsu_stores = store && (contiguous & 4);
#define CMB_TILE_CASE(S)                                                                      \
  case S:                                                                                     \
    if (lsu_stores) return launch_tile_lsu<S>(sm, shape, tile_bytes, dst, status, stream, grid); \
    return store ? launch_tile<S, true>(sm, dm, shape, tile_bytes, ctas_per_sm, status,       \
                                        xor_out, stream, grid)                                \
                 : launch_tile<S, false>(sm, dm, shape, tile_bytes, ctas_per_sm, status,      \
                                         xor_out, stream, grid);
  switch (stages) {
    CMB_TILE_CASE(2)
    CMB_TILE_CASE(3)
    CMB_TILE_CASE(4)
    CMB_TILE_CASE(5)
    CMB_TILE_CASE(6)
    CMB_TILE_CASE(7)
    CMB_TILE_CASE(8)
    default: break;
  }
#undef CMB_TILE_CASE
  return fail(CMB_ERR_INVALID_ARG, "tma tile: stages %d", stages);
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" int cmb_tma_tile_copy_bf16(void *dst, const void *src, int rows, int cols,
                                      int box_rows, int box_cols, int stages, int ctas_per_sm,
                                      int *status, cmb_stream_t stream) {
  if (dst == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_tma_tile_copy_bf16: null dst");
  return tile_impl(dst, src, rows, cols, box_rows, box_cols, stages, ctas_per_sm, status, nullptr,
                   0, 0, stream);
}

extern "C" int cmb_tma_tile_copy_tuned(void *dst, const void *src, int rows, int cols,
                                       int box_rows, int box_cols, int stages, int ctas_per_sm,
                                       int flags, int *status, cmb_stream_t stream) {
  if (dst == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_tma_tile_copy_tuned: null dst");
  return tile_impl(dst, src, rows, cols, box_rows, box_cols, stages, ctas_per_sm, status, nullptr,
                   0, flags, stream);
}

extern "C" int cmb_tma_tile_load_bf16(const void *src, int rows, int cols, int box_rows,
                                      int box_cols, int stages, uint32_t *xor_out,
                                      size_t xor_words, int *status, cmb_stream_t stream) {
  if (xor_out == nullptr || xor_words == 0)
    return fail(CMB_ERR_INVALID_ARG, "cmb_tma_tile_load_bf16: null xor_out");
  int grid = current_sm_count();
  if ((size_t)grid > xor_words) grid = static_cast<int>(xor_words);
  CMB_CUDA_TRY(cudaMemsetAsync(xor_out, 0, xor_words * sizeof(uint32_t), stream));
  return tile_impl(nullptr, src, rows, cols, box_rows, box_cols, stages, 1, status, xor_out, grid,
                   0, stream);
}

extern "C" int cmb_tma_1d_latency(const void *buf, size_t bytes, size_t offset, int iters,
                                  uint32_t *out_cycles, uint8_t *landed, int *status,
                                  cmb_stream_t stream) {
  if (buf == nullptr || out_cycles == nullptr || iters <= 0)
    return fail(CMB_ERR_INVALID_ARG, "cmb_tma_1d_latency: null buffer/output or iters <= 0");
  if (bytes < 16 || (reinterpret_cast<uintptr_t>(buf) & 15))
    return fail(CMB_ERR_INVALID_ARG, "cmb_tma_1d_latency: need >= 16 bytes, 16-byte aligned");
  // The load's x coordinate (bytes) must be 16-byte aligned, and the 16
  // bytes must lie inside the buffer.
  if ((offset & 15) != 0 || offset > bytes - 16 || offset > 0x7FFFFFF0u)
    return fail(CMB_ERR_INVALID_ARG,
                "cmb_tma_1d_latency: offset %zu not a multiple of 16 inside %zu bytes", offset,
                bytes);
  if (landed != nullptr && (reinterpret_cast<uintptr_t>(landed) & 15))
    return fail(CMB_ERR_INVALID_ARG, "cmb_tma_1d_latency: landed not 16-byte aligned");
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return fail(CMB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  CUtensorMap map;
  cuuint64_t dim[1] = {bytes};
  cuuint64_t stride[1] = {0};
  cuuint32_t box[1] = {16};
  cuuint32_t es[1] = {1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, const_cast<void *>(buf), dim, stride,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CMB_ERR_INVALID_ARG, "cuTensorMapEncodeTiled 1-D failed (%d)",
                                     static_cast<int>(r));
  if (status != nullptr) CMB_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), stream));
  k_tma_1d_latency<<<1, 32, 0, stream>>>(map, static_cast<int>(offset), iters, out_cycles, landed,
                                         status);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}
