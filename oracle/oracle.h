/*
 * oracle.h — CPU oracle for the probe path (TEST INFRASTRUCTURE ONLY).
 *
 * This is a plain-C restatement of what the reference suite's probe kernels
 * compute, used as the checker by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py.  Nothing in the product (the CUDA library,
 * the CLI, the Python package) links, loads or calls it.
 *
 * Parity status against the reference:
 *   - hash fill: restates the reference formula (src/mem_global.cu:7-10,
 *     include/memory_chase.h:128-133); pinned to the output of the
 *     reference's kernel_init_stream run on a B200.
 *   - chase endpoint: the reference's only self-check
 *     (include/memory_chase.h:152-153,161-164) is the walk restated in
 *     orc_chase_walk(); pinned to the endpoints of the reference's
 *     kernel_random_chase_cg run on a B200 over orc_chase_build's array.
 *   - stream sum, copy, TMA tile copy, GEMM: the reference pins no result for
 *     these (its outputs are XOR sinks, one smem byte, or sums of constants),
 *     so these restatements are parity unpinned against the reference; tests
 *     check them through size-independent properties (identity, fp64
 *     re-summation, fp64 GEMM on sampled tiles).
 * The fixtures and the scripts that made them are in tests/golden/
 * (make_golden.py: the reference's result logger; make_ref_fixtures.py: the
 * reference's kernels built for sm_100a by this directory's Makefile).
 */
#ifndef CMB_ORACLE_H
#define CMB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* SplitMix64: output i (0-based) of the stream seeded with `seed`. */
uint64_t orc_splitmix64_at(uint64_t seed, uint64_t i);

/* Reference hash fill: murmur3 fmix32 of (i + 0x9e3779b9)
 * (src/mem_global.cu:7-10, include/memory_chase.h:129-132). */
uint32_t orc_hash32(uint32_t i);
void orc_fill_hash_u32(uint32_t *out, size_t n);

/* fp32 uniform in [-1, 1): top 24 bits of SplitMix64 output i, scaled by
 * 2^-23, minus 1 (exact in fp32). */
void orc_fill_uniform_f32(float *out, size_t n, uint64_t seed);

/* Random bytes: byte i is byte (i % 8) (little endian) of output i / 8. */
void orc_fill_bytes(uint8_t *out, size_t n, uint64_t seed);

/* Pointer-chase link array over 128-byte slots (32 uint32 words per slot).
 * Word 0 of slot s holds the word index of the next slot; all other words
 * hold orc_hash32(word index).  The slot order is one Sattolo cycle drawn
 * from SplitMix64(seed).  Follows include/memory_chase.h:125-138 with the
 * shuffle replaced by Sattolo's algorithm. */
void orc_chase_build(uint32_t *links, size_t bytes, uint64_t seed);
/* Dependent walk idx = links[idx], `hops` times from `start`
 * (include/memory_chase.h:152-153). */
uint32_t orc_chase_walk(const uint32_t *links, uint64_t hops, uint32_t start);
/* 1 if following word-0 links from slot 0 visits every slot exactly once
 * before returning to slot 0. */
int orc_chase_is_single_cycle(const uint32_t *links, size_t bytes);

/* fp64 sum of fp32 values, blocked over `threads` host threads (<=0: all). */
double orc_sum_f64(const float *x, size_t n, int threads);
/* memcpy split across `threads` host threads; returns elapsed seconds. */
double orc_memcpy_mt(void *dst, const void *src, size_t n, int threads);
/* Host thread count that orc_* functions use for threads <= 0. */
int orc_hw_threads(void);

/* Number formats (OCP FP8 E4M3, bfloat16), round-to-nearest-even. */
float orc_bf16_to_f32(uint16_t v);
uint16_t orc_f32_to_bf16_rne(float f);
float orc_e4m3_to_f32(uint8_t v);
/* RNE with saturation to +-448 for finite inputs (the __NV_SATFINITE rule). */
uint8_t orc_f32_to_e4m3_satfinite(float f);

/* Per-tensor e4m3 quantisation: inv = 448 / amax (fp32), q = e4m3(x * inv). */
float orc_amax_bf16(const uint16_t *x, size_t n);
void orc_quantize_e4m3(const uint16_t *x, size_t n, float inv_scale, uint8_t *q);

/* fp64 reference for C = A * B^T on one tile.  A is M x K row-major, B is
 * N x K row-major (the "row.col" operand layout of
 * src/tensor_core_extended.cu:116), dtype 0 = bf16, 1 = e4m3 (scaled by
 * scale_a / scale_b).  out is tm x tn row-major. */
void orc_gemm_tile_f64(const void *A, const void *B, int dtype, int K,
                       int lda, int ldb, int row0, int col0, int tm, int tn,
                       double scale_a, double scale_b, double *out);
/* orc_gemm_tile_f64 on `ntiles` tiles at once over host threads (threads
 * <= 0: all).  tiles holds (row0, col0, tm, tn) per tile; the tiles' outputs
 * are stored one after another in out (tile t at the sum of the earlier
 * tiles' tm * tn), each tm x tn row-major.  Every output element is summed
 * in k order, as in orc_gemm_tile_f64. */
void orc_gemm_tiles_f64(const void *A, const void *B, int dtype, int K, int lda, int ldb,
                        int ntiles, const int *tiles, double scale_a, double scale_b,
                        double *out, int threads);
/* Blocked fp32 GEMM over host threads (the CPU baseline's timed kernel);
 * computes rows [row0, row0 + rows) of C = A * B^T for bf16 A, B, written
 * as a rows x N row-major block at C.  Threads split the output columns. */
void orc_gemm_bf16_rows_f32(const uint16_t *A, const uint16_t *B, float *C,
                            int N, int K, int row0, int rows, int threads);

#ifdef __cplusplus
}
#endif
#endif
