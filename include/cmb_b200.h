/*
 * cmb_b200.h — C ABI of the B200 (sm_100a) probe library libcmb_b200.so.
 *
 * The reference suite (cuda_micro_bench) has no FFI: its probe path is a set
 * of C++ functions `void cmb::benchmark_<section>()` that allocate, launch,
 * time and log inside one executable.  This header exposes the same path as
 * plain C entry points so any host (C, C++, Python ctypes, cgo, JNI) can
 * bind it: the kernels take device pointers and sizes and launch on the
 * caller's stream; the section entry points run a whole probe section and
 * log into the results table that cmb_results_write_json() writes in the
 * reference's results.json schema.
 *
 * Conventions
 *   - Every function returns a cmb_status (0 = CMB_OK).  On failure a
 *     one-line reason is available from cmb_last_error() (per thread).
 *   - Device pointers are plain pointers to device memory of the current
 *     device; host pointers say so in their name.
 *   - `stream` is a CUDA stream handle (cudaStream_t / CUstream); NULL is
 *     the legacy default stream.  Launch functions are asynchronous.
 *   - Kernels whose work is bounded by a device-side wait write a status
 *     word (cmb_status) to `status` (device int*, may be NULL) instead of
 *     hanging: CMB_ERR_TIMEOUT means a wait gave up.
 */
#ifndef CMB_B200_H
#define CMB_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *cmb_stream_t;

typedef enum {
  CMB_OK = 0,
  CMB_ERR_INVALID_ARG = 1,  /* bad size, alignment or pointer */
  CMB_ERR_CUDA = 2,         /* a CUDA runtime/driver call failed */
  CMB_ERR_TIMEOUT = 3,      /* a bounded device-side wait expired */
  CMB_ERR_UNSUPPORTED = 4,  /* device is not sm_100 or lacks a feature */
  CMB_ERR_MISMATCH = 5,     /* a probe's self-check failed */
  CMB_ERR_IO = 6            /* results file could not be written */
} cmb_status;

/* --- status -------------------------------------------------------- */

/* Name of a status code ("CMB_OK", ...). */
const char *cmb_status_string(int status);
/* Reason for the last failure on the calling thread ("" if none). */
const char *cmb_last_error(void);
/* Library version string. */
const char *cmb_version(void);
/* cudaDeviceReset() of the current device in the library's own CUDA
 * runtime, after releasing the streams and events the library keeps for
 * that device.  The library links the CUDA runtime statically, so a
 * caller's cudaDeviceReset() reaches only the caller's runtime; a process
 * that resets a device it used through this library calls this as well.
 * Every device allocation made through the library on that device is
 * gone afterwards.  No reference counterpart (the reference is one
 * executable with one runtime). */
int cmb_device_reset(void);

/* --- seeded input generators (not part of any timed region) ---------- */

/* dst[i] = fmix32(i + 0x9e3779b9): replaces kernel_init_stream
 * (src/mem_global.cu:5-12). */
int cmb_fill_hash_u32(uint32_t *dst, size_t n, cmb_stream_t stream);
/* dst[i] = uniform fp32 in [-1,1) from SplitMix64(seed) output i. */
int cmb_fill_uniform_f32(float *dst, size_t n, uint64_t seed, cmb_stream_t stream);
/* dst[i] = byte i%8 of SplitMix64(seed) output i/8. */
int cmb_fill_bytes(uint8_t *dst, size_t n, uint64_t seed, cmb_stream_t stream);
/* dst[i] = bf16(scale * N(0,1)), Box-Muller on SplitMix64(seed). */
int cmb_fill_normal_bf16(uint16_t *dst, size_t n, uint64_t seed, float scale,
                         cmb_stream_t stream);

/* --- global-memory streams (src/mem_global.cu) ----------------------- */

/* dst[0:bytes) = src[0:bytes).  Replaces kernel_stream_copy and its launch
 * (src/mem_global.cu:13-16,46).  Any size and alignment; 16-byte aligned
 * pointers take the vector path. */
int cmb_stream_copy(void *dst, const void *src, size_t bytes, cmb_stream_t stream);
/* cmb_stream_copy with an explicit launch shape, for sweeps: vec_bytes 16 or
 * 32, unroll 1/2/4/8 vectors in flight per thread, ctas_per_sm 1..8 CTAs of
 * 256 threads per SM. */
int cmb_stream_copy_tuned(void *dst, const void *src, size_t bytes, int vec_bytes, int unroll,
                          int ctas_per_sm, cmb_stream_t stream);

/* Workspace bytes cmb_stream_sum_f32 needs for n values. */
size_t cmb_stream_sum_workspace_bytes(size_t n);
/* *out_sum (device double) = sum of src[0:n) (fp32 loads, fp32 per-thread
 * partials, fp64 block and grid combine, fixed order).  Replaces the
 * read-only stream kernel_stream_read (src/mem_global.cu:17-26,47), whose
 * XOR sink is replaced by a checkable sum.  `workspace` is device memory of
 * cmb_stream_sum_workspace_bytes(n) bytes; it needs no initialisation.
 * Two calls whose work overlaps on the GPU need separate workspaces.  The
 * call enqueues two kernels: the sum, and a one-CTA combine launched with
 * programmatic stream serialization that writes *out_sum once the sum grid
 * has completed. */
int cmb_stream_sum_f32(const float *src, size_t n, double *out_sum, void *workspace,
                       size_t workspace_bytes, cmb_stream_t stream);

/* The same sum without a caller-supplied workspace, for callers that cannot
 * allocate device memory: code whose device memory is all owned by another
 * allocator (a framework's caching allocator or a fixed arena), or
 * latency-critical paths that cannot afford cudaMalloc/cudaFree, which may
 * synchronise the device.  No counterpart in the reference.
 * The workspace lives in a 33,024-byte array inside the library (one copy
 * on every GPU that loads it, kept until the process exits): room for
 * cmb_stream_sum_noalloc_max_ctas() = 4096 per-CTA partials.  The sum
 * launches up to 4 CTAs per SM, so any n fits on GPUs of up to 1024 SMs;
 * a GPU that would need more returns CMB_ERR_INVALID_ARG.  Nothing is
 * allocated: no cudaMalloc, cudaFree or allocating library call.
 * Every call looks up the array's device address in the current context
 * (cudaGetSymbolAddress), so a call after cmb_device_reset() uses the
 * reloaded array.  All calls on a device share the array: calls that
 * overlap on the GPU (other streams, or other host threads) race and give
 * wrong sums; serialise them.  The result equals cmb_stream_sum_f32's for
 * the same input. */
int cmb_stream_sum_f32_noalloc(const float *src, size_t n, double *out_sum, cmb_stream_t stream);
/* Capacity of that array in per-CTA partials (4096). */
size_t cmb_stream_sum_noalloc_max_ctas(void);

/* L2 aggregate read bandwidth: ctas CTAs (<= 0: 4 per SM) of 256 threads
 * read buf[0:bytes) `passes` times with 16-byte ld.global.cg (L1 bypassed;
 * size the buffer to stay in L2); *sum (device) = passes * (sum of the
 * buffer's 32-bit words) mod 2^64.  Replaces kernel_l2_aggregate_bw
 * (src/memory_more.cu:66-85), whose float sum is replaced by an exact one. */
int cmb_l2_read(const void *buf, size_t bytes, int passes, int ctas, unsigned long long *sum,
                cmb_stream_t stream);
/* The same exact sum with the bytes brought from L2 into shared memory by
 * cp.async.bulk (the TMA unit): one CTA per SM, twelve warps each streaming
 * 8 KiB chunks through a 2-stage ring (lane 0 loads, the warp adds the
 * words).  bytes a positive multiple of 8 KiB; *status (device, may be
 * NULL) = CMB_ERR_TIMEOUT if a chunk never landed within 2 s.  No reference
 * counterpart (the reference reads L2 with register loads only). */
int cmb_l2_read_bulk(const void *buf, size_t bytes, int passes, unsigned long long *sum,
                     int *status, cmb_stream_t stream);

/* Host-buffer stream copy: host_dst = host_src through the device.  Copies
 * chunks host->device, runs cmb_stream_copy on each, copies them back, with
 * the three steps of consecutive chunks overlapped on three streams.
 * dev_a/dev_b are device staging buffers of dev_bytes each (dev_bytes >=
 * 2*chunk); host buffers should be pinned for full speed.  Blocks until
 * host_dst is complete. */
int cmb_stream_copy_host(void *host_dst, const void *host_src, size_t bytes, void *dev_a,
                         void *dev_b, size_t dev_bytes, size_t chunk);

/* --- dependent-load pointer chase (src/memory_chase.cu,
 *     include/memory_chase.h) ------------------------------------------ */

/* Host: fill host_links (bytes/4 words) with one Sattolo cycle over the
 * bytes/128 slots of 128 B (word 0 of each slot links to the next slot's
 * word index; the other words hold fmix32 of their index).  Replaces the
 * host cycle build of measureRandomChase (include/memory_chase.h:125-138). */
int cmb_chase_build_links(uint32_t *host_links, size_t bytes, uint64_t seed);

/* One thread follows idx = links[idx] from word 0: `warmup` untimed hops,
 * then `hops` timed hops.  bypass_l1 = 1 uses ld.global.cg, 0 uses
 * ld.global.ca.  out (device, 4 x uint64) = {SM cycles of the timed hops,
 * final index, globaltimer ns of the timed hops, status}; status is
 * CMB_ERR_INVALID_ARG (and the walk is skipped) if a slot head of the
 * `words`-word array is not an in-range slot index.  Replaces
 * kernel_random_chase_cg/_ca (src/memory_chase.cu:6-34). */
int cmb_chase_run(const uint32_t *links, size_t words, uint64_t warmup, uint64_t hops,
                  int bypass_l1, uint64_t *out, cmb_stream_t stream);

/* Host: *out_index = the index reached after `hops` hops of idx =
 * host_links[idx] from 0, the expected endpoint of cmb_chase_run with
 * warmup + hops = `hops` (the reference's self-check,
 * include/memory_chase.h:152-153,161-164).  CMB_ERR_INVALID_ARG if the walk
 * leaves the array. */
int cmb_chase_host_walk(const uint32_t *host_links, size_t words, uint64_t hops,
                        uint32_t *out_index);

/* --- TMA bulk-tensor tile movement (src/tma.cu) --------------------- */

/* dst = src for a rows x cols row-major bf16 matrix, moved in box_rows x
 * box_cols tiles by cp.async.bulk.tensor loads into a `stages`-deep
 * shared-memory ring (mbarrier complete_tx) and tiled TMA stores back out;
 * ctas_per_sm persistent CTAs per SM stride over the tiles.  Needs cols % 8
 * == 0, 16-byte aligned bases, box dims in [1,256] x [8,256] with box bytes
 * a multiple of 1024 and stages * box bytes <= 226 KiB.  Replaces
 * kernel_tma_g2s_bandwidth (src/tma.cu:72-121), which loaded 16 KiB bulk
 * chunks and discarded them, with a verifiable tile copy. */
int cmb_tma_tile_copy_bf16(void *dst, const void *src, int rows, int cols, int box_rows,
                           int box_cols, int stages, int ctas_per_sm, int *status,
                           cmb_stream_t stream);
/* cmb_tma_tile_copy_bf16 with placement options, for sweeps: flags bit 0 =
 * give each CTA one contiguous run of tiles (default: CTA b strides over
 * tiles b, b + grid, ... in row-major tile order); bit 1 = L2 evict-first
 * policy on the loads and stores (TMA stores only); bit 2 = write the tiles
 * with load/store-unit stores from 4 warps instead of TMA stores (the stage
 * returns to the loads once read into registers). */
int cmb_tma_tile_copy_tuned(void *dst, const void *src, int rows, int cols, int box_rows,
                            int box_cols, int stages, int ctas_per_sm, int flags, int *status,
                            cmb_stream_t stream);
/* Load-only form of the same pipeline (the reference's read-only G2S
 * bandwidth, src/tma.cu:72-121,247): one CTA per SM (at most xor_words);
 * CTA b writes to xor_out[b] the XOR of the first four 32-bit words of every
 * tile it loaded (tiles b, b + grid, ...; the other entries are zeroed). */
int cmb_tma_tile_load_bf16(const void *src, int rows, int cols, int box_rows, int box_cols,
                           int stages, uint32_t *xor_out, size_t xor_words, int *status,
                           cmb_stream_t stream);
/* One thread issues `iters` 16-byte 1-D TMA loads of buf[offset:offset+16)
 * into the same zeroed shared-memory slot, waiting for each; *out_cycles
 * (device) = SM cycles of the loop; landed (device, 16 bytes, 16-byte
 * aligned, may be NULL) = the 16 bytes in shared memory after the last
 * load, which must equal buf[offset:offset+16).  offset is a multiple of
 * 16 with offset + 16 <= bytes (the TMA coordinate's alignment rule).
 * Replaces kernel_tma_1d_latency (src/tma.cu:20-69), which loads from
 * coordinate 0 and keeps no output. */
int cmb_tma_1d_latency(const void *buf, size_t bytes, size_t offset, int iters,
                       uint32_t *out_cycles, uint8_t *landed, int *status, cmb_stream_t stream);

/* --- tcgen05 dense GEMM (src/tensor_core.cu, src/tensor_core_extended.cu)  */

/* C[M x N] (fp32, row-major) = A[M x K] * B[N x K]^T for bf16 A, B stored
 * K-major (row-major with K contiguous; the "row.col" operand order of
 * src/tensor_core_extended.cu:116), fp32 accumulation in tensor memory.
 * cta_group 1: 128 x 256 tiles per CTA; 2: 256 x 512 tiles per pair of CTAs
 * (cta_group::2 MMAs, two N = 256 accumulators filling TMEM).  Needs K % 8 == 0 and 16-byte aligned A, B.
 * Replaces the register-only mma.sync throughput kernels
 * (src/tensor_core_extended.cu:77-128,265-292) with a GEMM that reads and
 * writes memory and has a checkable result. */
int cmb_gemm_bf16(const void *A, const void *B, float *C, int M, int N, int K, int cta_group,
                  int *status, cmb_stream_t stream);
/* Same for e4m3 A, B (K % 16 == 0): C = (*scale_a) * (*scale_b) * A * B^T,
 * scales read from device memory.  Replaces the FP8 mma.sync kernels
 * (src/tensor_core_extended.cu:133-184). */
int cmb_gemm_e4m3(const void *A, const void *B, float *C, int M, int N, int K,
                  const float *scale_a, const float *scale_b, int cta_group, int *status,
                  cmb_stream_t stream);
/* cmb_gemm_bf16 (fp8 = 0) or cmb_gemm_e4m3 (fp8 = 1) with an explicit
 * pipeline shape, for sweeps: stages 3-4 (cta_group 1) or 4-6 (cta_group 2;
 * 7 with epilogue 1), 0 = default (4); group_m = tile rows per raster
 * group, 0 = default (8); epilogue 1 = direct stores, 2 = TMA stores (needs
 * N % 4 == 0), 0 = default (2 when possible); tile_n = output columns per
 * tile, 256 or (cta_group 2, stages 3-4) 512 = two N=256 MMAs per K slice
 * into all 512 TMEM columns, 0 = default (512 for cta_group 2, else 256);
 * epi_warps = epilogue warps, 4 or (tile_n 512, stages 3-4) 8 = each warp
 * drains 128 columns of one N=256 half through registers and the half is
 * handed back to the next tile's MMAs before it is stored, 0 = default
 * (8 for tile_n 512, else 4). */
int cmb_gemm_tuned(const void *A, const void *B, float *C, int M, int N, int K, int fp8,
                   const float *scale_a, const float *scale_b, int cta_group, int stages,
                   int group_m, int epilogue, int tile_n, int epi_warps, int *status,
                   cmb_stream_t stream);
/* cmb_gemm_bf16 (fp8 = 0) or cmb_gemm_e4m3 (fp8 = 1) with a bf16 C: each fp32
 * accumulator (times *scale_a * *scale_b for e4m3) is rounded to the nearest
 * bf16, ties to even.  2-CTA 256 x 512 tiles with the held epilogue; TMA
 * stores of 32 x 64 boxes when N % 8 == 0 and C is 16-byte aligned, direct
 * stores otherwise.  No reference counterpart (its probes store nothing);
 * the output type of the measured cuBLAS peak. */
int cmb_gemm_bf16_out(const void *A, const void *B, void *C, int M, int N, int K, int fp8,
                      const float *scale_a, const float *scale_b, int *status,
                      cmb_stream_t stream);
/* Tensor-pipe ceiling: `ctas` CTAs (one per SM) each issue `iters` rounds of
 * four tcgen05.mma M=128 N=256 (bf16: fp8 = 0, K = 16; e4m3: fp8 = 1,
 * K = 32) on all-ones operands resident in shared memory, into TMEM, with no
 * other memory traffic.  out (device, ctas * 128 floats) = one accumulator
 * value per row, each iters * 4 * K (status CMB_ERR_MISMATCH if any checked
 * element differs); cycles (device, ctas x uint64, may be NULL) = SM cycles
 * of each CTA's issue loop.  The tcgen05 counterpart of the register-only
 * mma.sync throughput kernels (src/tensor_core_extended.cu:170-250). */
int cmb_mma_rate(int fp8, int iters, int ctas, float *out, uint64_t *cycles, int *status,
                 cmb_stream_t stream);
/* Per-tensor e4m3 quantisation of n bf16 values: amax = max |x|,
 * dst[i] = e4m3_satfinite(x[i] * (448 / amax)) (fp32 multiply, round to
 * nearest even), scale_out[0] = amax / 448 (the dequantisation factor),
 * scale_out[1] = amax; scale_out is device memory of 2 floats. */
int cmb_quantize_e4m3(const uint16_t *src_bf16, size_t n, uint8_t *dst, float *scale_out,
                      cmb_stream_t stream);

/* --- die-aware tile order for the GEMMs (no reference counterpart: the
 *     reference's tensor probes read no memory) ---------------------------- */

/* Size of a per-SM die map: one entry per %smid value. */
#define CMB_DIE_MAP_IDS 256
/* Measures which of the B200's two dies each SM of the current device sits
 * on: after L2 is evicted, each SM in turn times cold loads of the same 96
 * lines; a line homed on the other die's memory takes a die crossing more,
 * so SMs of one die share a near/far pattern.  sm_die[id] (host, capacity
 * entries) = 0 or 1 for every SM id (die 0 holds the lowest id), 0xFF for
 * ids no SM has; *n_ids = highest SM id + 1.  near_far_cycles (host, 2
 * floats, may be NULL) = median cold-load latency near and far.  Runs ~300
 * short launches on `stream` (tens of ms), allocates and frees 288 MiB of
 * device memory, and needs the device otherwise idle (every SM must take
 * one of its CTAs).  CMB_ERR_MISMATCH when the SMs do not split cleanly in
 * two (after a second measurement). */
int cmb_sm_die_map(uint8_t *sm_die, int capacity, int *n_ids, float *near_far_cycles,
                   cmb_stream_t stream);
/* Installs a die map (as cmb_sm_die_map returns it: n_ids entries of 0, 1
 * or 0xFF, both dies non-empty) for the GEMMs that later launch on the
 * current device: their tiles are cut into one contiguous range per die,
 * in proportion to its SMs, and each CTA cluster works in its own die's
 * range, so less operand data crosses between the dies.  The result is
 * bit-identical with or without a map, and with any map: the map only moves
 * tiles between clusters.  sm_die == NULL or n_ids == 0 removes the map
 * (the plain persistent order).  Copies the map to the device
 * synchronously: call it while no GEMM of this library runs on the device.
 * Up to 64 GEMM launches may run on one device at the same time. */
int cmb_gemm_set_sm_die_map(const uint8_t *sm_die, int n_ids);

/* --- legacy warp-level mma.sync probes (src/tensor_core.cu,
 *     src/tensor_core_extended.cu) ------------------------------------- */

/* kind: 0 = tf32 m16n8k8 (f32 acc), 1 = f16 m16n8k16 (f16 acc), 2 = bf16
 * m16n8k16 (f32 acc), 3 = e4m3 m16n8k32 (f32 acc), 4 = s8 m16n8k32 (s32 acc);
 * all operands 1.  Latency: one warp runs a dependent chain of `iters` MMAs;
 * *cycles (device) = SM cycles of the chain, *value (device) = accumulator
 * element 0 (iters * K; f16 saturates).  Replaces kernel_mma_latency and
 * kernel_hmma_*_latency (src/tensor_core.cu:13-39,
 * src/tensor_core_extended.cu:21-46,77-102,133-158,189-214). */
int cmb_mma_sync_latency(int kind, int iters, uint64_t *cycles, double *value,
                         cmb_stream_t stream);
/* Throughput: blocks x warps_per_block warps each run four independent
 * chains of `iters` MMAs; values (device, one double per warp) = sum of the
 * four chains' element 0.  Replaces kernel_mma_throughput and
 * kernel_hmma_*_throughput (src/tensor_core.cu:41-64,
 * src/tensor_core_extended.cu:48-72,104-128,160-184,216-240). */
int cmb_mma_sync_throughput(int kind, int iters, int blocks, int warps_per_block,
                            double *values, cmb_stream_t stream);

/* --- multi-GPU: NVLink peer copies (new; the reference only queries
 *     cudaDeviceCanAccessPeer, src/pcie.cu:100-112) -------------------- */

/* Device buffers that peers may map: plain cudaMalloc / cudaFree (an IPC
 * handle must name the start of an allocation). */
int cmb_p2p_alloc(size_t bytes, void **out);
int cmb_p2p_free(void *ptr);
/* Bytes of an IPC handle (64). */
size_t cmb_ipc_handle_bytes(void);
/* handle_out (host, cmb_ipc_handle_bytes() bytes) names the allocation that
 * starts at `base` (from cmb_p2p_alloc), for another process to open. */
int cmb_ipc_get_handle(void *base, void *handle_out);
/* Maps another process's allocation into this one (peer access enabled on
 * first use); *peer_ptr is a device pointer usable by this GPU's kernels and
 * copy engines. */
int cmb_ipc_open(const void *handle, void **peer_ptr);
int cmb_ipc_close(void *peer_ptr);
/* One process driving several GPUs: lets the current device access
 * `peer_device`'s memory (no error if already enabled). */
int cmb_p2p_enable_peer(int peer_device);
/* n (1..8) copies dst[j][0:bytes[j]) = src[j][0:bytes[j]) in one kernel:
 * SMs of the current GPU load src (its own memory) and store to dst, which
 * may be another GPU's memory (peer stores over NVLink).  16-byte aligned
 * pointers; ctas_per_job <= 0 picks 2 * SMs / n. */
int cmb_p2p_scatter_store(void *const *dst, const void *const *src, const size_t *bytes, int n,
                          int ctas_per_job, cmb_stream_t stream);
/* cmb_p2p_scatter_store with an explicit vector width (16 or 32 bytes;
 * pointers aligned to it), for sweeps.  cmb_p2p_scatter_store uses 32 when
 * every job is 32-byte aligned. */
int cmb_p2p_scatter_store_tuned(void *const *dst, const void *const *src, const size_t *bytes,
                                int n, int ctas_per_job, int vec_bytes, cmb_stream_t stream);
/* The same n copies by cp.async.bulk: one thread per CTA streams 16 KiB
 * chunks of src (this GPU's memory) through an 8-stage shared-memory ring
 * and writes each chunk to dst (which may be a peer's memory) with one bulk
 * store.  16-byte aligned pointers; ctas_per_job <= 0 picks 32 (at most
 * SMs / n), which on a ring reach the same NVLink rate as peer stores from
 * every SM; *status (device, may be NULL) = CMB_ERR_TIMEOUT if a chunk
 * load never completed within 2 s.  After such a timeout a CTA issues no
 * further loads and waits up to 0.1 s for each load still in flight; if one
 * of those never lands either, the CTA exits with it outstanding, so a
 * CMB_ERR_TIMEOUT from this call means the context must be treated as
 * unusable (reset the device).  No reference counterpart (new NVLink
 * probe). */
int cmb_p2p_scatter_bulk(void *const *dst, const void *const *src, const size_t *bytes, int n,
                         int ctas_per_job, int *status, cmb_stream_t stream);
/* cmb_p2p_scatter_bulk with an explicit chunk size (multiple of 16, at most
 * 64 KiB, 0 = 16 KiB) and ring depth (4 stages with 2 stores in flight, or 8
 * with 4; 0 = 8; stages x chunk <= 227 KiB), for sweeps. */
int cmb_p2p_scatter_bulk_tuned(void *const *dst, const void *const *src, const size_t *bytes,
                               int n, int ctas_per_job, int chunk_bytes, int stages, int *status,
                               cmb_stream_t stream);
/* The same n copies by the copy engines (cudaMemcpyAsync, one internal
 * stream per job, joined back into `stream`). */
int cmb_p2p_scatter_copy_engine(void *const *dst, const void *const *src, const size_t *bytes,
                                int n, cmb_stream_t stream);
/* cmb_p2p_scatter_copy_engine over `streams` (1..8) internal streams: job j
 * runs on stream j % streams, after the earlier jobs of that stream, so the
 * order of the jobs is the order each stream visits its destinations (an
 * all-to-all whose ranks start at different peers keeps every receiver
 * busy with one sender at a time). */
int cmb_p2p_scatter_copy_engine_tuned(void *const *dst, const void *const *src,
                                      const size_t *bytes, int n, int streams,
                                      cmb_stream_t stream);
/* The same n copies by both engines at once: the first ce_permille / 1000
 * of each job (rounded down to 4 KiB) by the copy engines on `ce_streams`
 * (1..8) internal streams as in cmb_p2p_scatter_copy_engine_tuned, the
 * rest by the SMs' peer stores as in cmb_p2p_scatter_store, both forked
 * from and joined back into `stream`.  16-byte aligned pointers. */
int cmb_p2p_scatter_hybrid(void *const *dst, const void *const *src, const size_t *bytes, int n,
                           int ce_permille, int ce_streams, cmb_stream_t stream);

/* --- self-test of the bounded-wait rule -------------------------------- */

/* One thread waits on an mbarrier phase that nothing completes, giving up
 * after limit_ns (<= 2 s): *status (device) = CMB_ERR_TIMEOUT and
 * *waited_ns (device) = how long it waited.  The device stays usable. */
int cmb_selftest_wait_timeout(uint64_t limit_ns, int *status, uint64_t *waited_ns,
                              cmb_stream_t stream);

/* --- checks ---------------------------------------------------------- */

/* *mismatches (device) = 0 iff a[0:bytes) == b[0:bytes) (otherwise the
 * number of differing 32-bit words, or bytes when a or b is not 16-byte
 * aligned). */
int cmb_compare_bytes(const void *a, const void *b, size_t bytes,
                      unsigned long long *mismatches, cmb_stream_t stream);

/* --- probe sections (src/main.cu:9-32) --------------------------------
 * Each runs one section on device 0 like the reference's
 * `void cmb::benchmark_<section>()`: allocates, checks outputs, times, and
 * logs into the results table under the reference's keys (plus new ones);
 * returns a status instead of exiting.
 * The library also exports, with C++ linkage, the reference's own
 *   void cmb::benchmark_global_memory(), cmb::benchmark_cache(),
 *   cmb::benchmark_tma(), cmb::benchmark_tensor_core(),
 *   cmb::benchmark_tensor_core_extended(), cmb::benchmark_multi_gpu()
 * (src/main.cu:9-32), which exit(EXIT_FAILURE) on a failure as the
 * reference's sections do, so the reference's main.cu links against the
 * library in place of its mem_global.cu, memory_chase.cu, mem_cache.cu,
 * tma.cu, tensor_core.cu and tensor_core_extended.cu.  No other C++ symbol
 * is exported. */
int cmb_benchmark_global_memory(void);       /* src/mem_global.cu:27-75 */
int cmb_benchmark_cache(void);               /* src/mem_cache.cu:4-24 */
int cmb_benchmark_tma(void);                 /* src/tma.cu:157-259 */
int cmb_benchmark_tensor_core(void);         /* src/tensor_core.cu:66-120 */
int cmb_benchmark_tensor_core_extended(void);  /* src/tensor_core_extended.cu:321-357 */
int cmb_benchmark_multi_gpu(void);           /* new: NVLink P2P and sharded stream */
int cmb_benchmark_memory_more(void);         /* src/memory_more.cu:201-234 (L2 bandwidth only) */
int cmb_benchmark_pcie(void);                /* src/pcie.cu:55-97 (pinned bandwidth only) */
/* Logs "N/A" for every key the reference's results/report.html reads that
 * no section logged, so the report renders. */
int cmb_results_log_report_placeholders(void);
/* The same key table, read-only: how many (section, key) paths the report
 * reads, and path i as two static strings.  No reference counterpart (the
 * reference keeps these paths only inside results/report.html). */
size_t cmb_report_key_count(void);
int cmb_report_key(size_t i, const char **section, const char **key);
/* The CLI (src/main.cu:156-181) with results written to json_path (NULL:
 * results/results.json); returns the process exit code. */
int cmb_run_cli(int argc, const char *const *argv, const char *json_path);

/* --- results table (include/result_logger.h, src/result_logger.cu) --- */

/* Same meaning as ResultLogger::setDevice (include/result_logger.h:113-121). */
int cmb_results_set_device(const char *name, const char *arch, int sm_count, int clock_khz,
                           int mem_clock_khz, int mem_bus_width);
/* Same meaning as ResultLogger::log (include/result_logger.h:123-126); unit
 * "N/A" writes a null value. */
int cmb_results_log(const char *section, const char *key, double value, const char *unit);
/* Writes the table in the reference's results.json format
 * (src/result_logger.cu:10-43). */
int cmb_results_write_json(const char *path);
/* Empties the table and the device fields. */
int cmb_results_clear(void);

/* Callbacks that receive every entry the library's table receives. */
typedef void (*cmb_results_log_fn)(const char *section, const char *key, double value,
                                   const char *unit, void *user);
typedef void (*cmb_results_device_fn)(const char *name, const char *arch, int sm_count,
                                      int clock_khz, int mem_clock_khz, int mem_bus_width,
                                      void *user);
/* From now on every ResultLogger::log / setDevice the library makes (its
 * sections and cmb_results_log / cmb_results_set_device) is also passed to
 * `log` / `device` (either may be NULL; both NULL uninstalls), one call at a
 * time, on the thread that logged.  This is how the library's sections log
 * into the reference's own cmb::g_results (include/result_logger.h:111-144)
 * when it is linked into the reference's main.cu: the library keeps its own
 * table private, and a shim in the reference build forwards each call to
 * g_results.log() and g_results.setDevice().  The callbacks must not call
 * the library's cmb_results_* functions.  No reference counterpart. */
int cmb_results_set_sink(cmb_results_log_fn log, cmb_results_device_fn device, void *user);

#ifdef __cplusplus
}
#endif
#endif /* CMB_B200_H */
