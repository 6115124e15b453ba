/*
 * oracle.c — CPU oracle for the probe path (TEST INFRASTRUCTURE ONLY; see
 * oracle.h).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline load this file's library.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

/* ------------------------------------------------------------------ */
/* generators                                                          */
/* ------------------------------------------------------------------ */

static const uint64_t kGolden = 0x9E3779B97F4A7C15ULL;

static inline uint64_t mix64(uint64_t z) {
  /* SplitMix64 output function (Steele, Lea, Flood 2014). */
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

uint64_t orc_splitmix64_at(uint64_t seed, uint64_t i) {
  return mix64(seed + (i + 1) * kGolden);
}

uint32_t orc_hash32(uint32_t i) {
  /* src/mem_global.cu:7-10 */
  uint32_t x = i + 0x9e3779b9U;
  x = (x ^ (x >> 16)) * 0x85ebca6bU;
  x = (x ^ (x >> 13)) * 0xc2b2ae35U;
  return x ^ (x >> 16);
}

void orc_fill_hash_u32(uint32_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_hash32((uint32_t)i);
}

void orc_fill_uniform_f32(float *out, size_t n, uint64_t seed) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t u = (uint32_t)(orc_splitmix64_at(seed, i) >> 40);
    out[i] = (float)u * 0x1p-23f - 1.0f;
  }
}

void orc_fill_bytes(uint8_t *out, size_t n, uint64_t seed) {
  for (size_t i = 0; i < n; ++i) {
    uint64_t w = orc_splitmix64_at(seed, i >> 3);
    out[i] = (uint8_t)(w >> (8 * (i & 7)));
  }
}

/* ------------------------------------------------------------------ */
/* pointer chase                                                       */
/* ------------------------------------------------------------------ */

void orc_chase_build(uint32_t *links, size_t bytes, uint64_t seed) {
  const size_t words = bytes / 4, slots = bytes / 128;
  for (size_t w = 0; w < words; ++w) links[w] = orc_hash32((uint32_t)w);
  if (slots == 0) return;
  uint32_t *perm = (uint32_t *)malloc(slots * sizeof(uint32_t));
  for (size_t s = 0; s < slots; ++s) perm[s] = (uint32_t)s;
  /* Sattolo: for i = n-1 .. 1, swap perm[i] with perm[j], j uniform in
   * [0, i).  Draw k of the SplitMix64 stream picks j for step k. */
  uint64_t k = 0;
  for (size_t i = slots - 1; i >= 1; --i, ++k) {
    uint64_t r = orc_splitmix64_at(seed, k);
    size_t j = (size_t)(((unsigned __int128)r * (uint64_t)i) >> 64);
    uint32_t t = perm[i];
    perm[i] = perm[j];
    perm[j] = t;
  }
  /* perm is one n-cycle; slot s links to slot perm[s]. */
  for (size_t s = 0; s < slots; ++s) links[s * 32] = perm[s] * 32u;
  free(perm);
}

uint32_t orc_chase_walk(const uint32_t *links, uint64_t hops, uint32_t start) {
  uint32_t idx = start;
  for (uint64_t h = 0; h < hops; ++h) idx = links[idx];
  return idx;
}

int orc_chase_is_single_cycle(const uint32_t *links, size_t bytes) {
  const size_t slots = bytes / 128;
  if (slots == 0) return 0;
  uint8_t *seen = (uint8_t *)calloc(slots, 1);
  uint32_t idx = 0;
  size_t count = 0;
  int ok = 1;
  do {
    if (idx % 32 != 0 || idx / 32 >= slots || seen[idx / 32]) { ok = 0; break; }
    seen[idx / 32] = 1;
    ++count;
    idx = links[idx];
  } while (idx != 0);
  free(seen);
  return ok && count == slots;
}

/* ------------------------------------------------------------------ */
/* threaded sum / memcpy                                               */
/* ------------------------------------------------------------------ */

int orc_hw_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static int pick_threads(int threads) {
  int t = threads > 0 ? threads : orc_hw_threads();
  return t > 256 ? 256 : t;
}

typedef struct {
  const float *x;
  size_t begin, end;
  double out;
} sum_job;

static void *sum_worker(void *p) {
  sum_job *j = (sum_job *)p;
  /* Blocks of 4096 values summed in fp64, then the block sums in fp64. */
  double acc = 0.0;
  for (size_t b = j->begin; b < j->end; b += 4096) {
    size_t e = b + 4096 < j->end ? b + 4096 : j->end;
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    size_t i = b;
    for (; i + 4 <= e; i += 4) {
      s0 += j->x[i];
      s1 += j->x[i + 1];
      s2 += j->x[i + 2];
      s3 += j->x[i + 3];
    }
    for (; i < e; ++i) s0 += j->x[i];
    acc += (s0 + s1) + (s2 + s3);
  }
  j->out = acc;
  return NULL;
}

double orc_sum_f64(const float *x, size_t n, int threads) {
  int t = pick_threads(threads);
  if ((size_t)t > n / 4096 + 1) t = (int)(n / 4096 + 1);
  pthread_t th[256];
  sum_job jobs[256];
  size_t per = (n + t - 1) / t;
  for (int k = 0; k < t; ++k) {
    jobs[k].x = x;
    jobs[k].begin = (size_t)k * per < n ? (size_t)k * per : n;
    jobs[k].end = (size_t)(k + 1) * per < n ? (size_t)(k + 1) * per : n;
    pthread_create(&th[k], NULL, sum_worker, &jobs[k]);
  }
  double total = 0.0;
  for (int k = 0; k < t; ++k) {
    pthread_join(th[k], NULL);
    total += jobs[k].out;
  }
  return total;
}

typedef struct {
  char *dst;
  const char *src;
  size_t n;
} copy_job;

static void *copy_worker(void *p) {
  copy_job *j = (copy_job *)p;
  memcpy(j->dst, j->src, j->n);
  return NULL;
}

double orc_memcpy_mt(void *dst, const void *src, size_t n, int threads) {
  int t = pick_threads(threads);
  pthread_t th[256];
  copy_job jobs[256];
  size_t per = ((n + t - 1) / t + 63) & ~(size_t)63;
  struct timespec a, b;
  clock_gettime(CLOCK_MONOTONIC, &a);
  int used = 0;
  for (int k = 0; k < t; ++k) {
    size_t off = (size_t)k * per;
    if (off >= n) break;
    jobs[k].dst = (char *)dst + off;
    jobs[k].src = (const char *)src + off;
    jobs[k].n = off + per <= n ? per : n - off;
    pthread_create(&th[k], NULL, copy_worker, &jobs[k]);
    ++used;
  }
  for (int k = 0; k < used; ++k) pthread_join(th[k], NULL);
  clock_gettime(CLOCK_MONOTONIC, &b);
  return (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
}

/* ------------------------------------------------------------------ */
/* number formats                                                      */
/* ------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float bf16_to_f32(uint16_t v) { return u2f((uint32_t)v << 16); }
float orc_bf16_to_f32(uint16_t v) { return bf16_to_f32(v); }

uint16_t orc_f32_to_bf16_rne(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))
    return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

/* OCP 8-bit floating point, E4M3: bias 7, no infinities, S.1111.111 = NaN,
 * largest finite 448, smallest subnormal 2^-9. */
float orc_e4m3_to_f32(uint8_t v) {
  int s = v >> 7, e = (v >> 3) & 0xf, m = v & 7;
  float mag;
  if (e == 0xf && m == 7) return NAN;
  if (e == 0) mag = ldexpf((float)m, -9);
  else mag = ldexpf((float)(8 + m), e - 10);
  return s ? -mag : mag;
}

uint8_t orc_f32_to_e4m3_satfinite(float f) {
  uint8_t sign = (f2u(f) >> 31) ? 0x80 : 0x00;
  if (isnan(f)) return 0x7f;
  float a = fabsf(f);
  if (a >= 448.0f) return sign | 0x7e; /* saturate (inf included) */
  /* Candidates are the 127 finite non-negative codes; pick the nearest,
   * ties to the even code (even mantissa LSB). */
  /* Quantum in the binade of a: normal e in [1,15] covers [2^-6, 2^9). */
  double x = (double)a;
  int code;
  if (x < 0x1p-6) {
    /* subnormal grid: multiples of 2^-9, codes 0..7 (8 = 2^-6 normal) */
    double q = x * 512.0; /* exact */
    double r = nearbyint(q); /* default rounding mode: ties to even */
    code = (int)r; /* 0..8; 8 is the smallest normal (e=1, m=0) */
  } else {
    int e;
    frexp(x, &e); /* x = f * 2^e, f in [0.5, 1) */
    int ub = e - 1; /* unbiased exponent, x in [2^ub, 2^(ub+1)) */
    double q = ldexp(x, 3 - ub); /* in [8, 16) */
    double r = nearbyint(q);
    int m = (int)r - 8; /* 0..8; 8 means carry into the next binade */
    int be = ub + 7;
    if (m == 8) { m = 0; be += 1; }
    code = (be << 3) | m;
    if (code > 0x7e) code = 0x7e;
  }
  return sign | (uint8_t)code;
}

float orc_amax_bf16(const uint16_t *x, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float a = fabsf(orc_bf16_to_f32(x[i]));
    if (a > m) m = a;
  }
  return m;
}

void orc_quantize_e4m3(const uint16_t *x, size_t n, float inv_scale, uint8_t *q) {
  for (size_t i = 0; i < n; ++i) {
    float v = orc_bf16_to_f32(x[i]) * inv_scale; /* one fp32 RN multiply */
    q[i] = orc_f32_to_e4m3_satfinite(v);
  }
}

/* ------------------------------------------------------------------ */
/* GEMM                                                                */
/* ------------------------------------------------------------------ */

void orc_gemm_tile_f64(const void *A, const void *B, int dtype, int K, int lda,
                       int ldb, int row0, int col0, int tm, int tn,
                       double scale_a, double scale_b, double *out) {
  double *arow = (double *)malloc((size_t)K * sizeof(double));
  double *bt = (double *)malloc((size_t)tn * K * sizeof(double));
  for (int j = 0; j < tn; ++j)
    for (int k = 0; k < K; ++k) {
      size_t o = (size_t)(col0 + j) * ldb + k;
      bt[(size_t)j * K + k] =
          dtype == 0 ? (double)orc_bf16_to_f32(((const uint16_t *)B)[o])
                     : (double)orc_e4m3_to_f32(((const uint8_t *)B)[o]) * scale_b;
    }
  for (int i = 0; i < tm; ++i) {
    for (int k = 0; k < K; ++k) {
      size_t o = (size_t)(row0 + i) * lda + k;
      arow[k] = dtype == 0 ? (double)orc_bf16_to_f32(((const uint16_t *)A)[o])
                           : (double)orc_e4m3_to_f32(((const uint8_t *)A)[o]) * scale_a;
    }
    for (int j = 0; j < tn; ++j) {
      const double *b = bt + (size_t)j * K;
      double s = 0.0;
      for (int k = 0; k < K; ++k) s += arow[k] * b[k];
      out[(size_t)i * tn + j] = s;
    }
  }
  free(arow);
  free(bt);
}

/* Sampled-tile check (orc_gemm_tiles_f64): the tile's B columns are decoded
 * once into k-major doubles, then threads take blocks of four output rows;
 * each block keeps 4 x 32 accumulators and walks k in order, so every
 * element is the same k-ordered sum orc_gemm_tile_f64 forms. */
typedef struct {
  const void *A;
  const double *bt; /* K x tn, k-major */
  double *out;
  int dtype, K, lda, row0, tm, tn;
  double scale_a;
  int next; /* next row block, taken under mu */
  pthread_mutex_t mu;
} tiles_job;

__attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
static void *tiles_worker(void *p) {
  tiles_job *g = (tiles_job *)p;
  enum { RB = 4, CB = 32 };
  const int K = g->K;
  double *a = (double *)malloc(sizeof(double) * RB * (size_t)K);
  for (;;) {
    pthread_mutex_lock(&g->mu);
    const int r0 = g->next;
    g->next += RB;
    pthread_mutex_unlock(&g->mu);
    if (r0 >= g->tm) break;
    const int rb = g->tm - r0 < RB ? g->tm - r0 : RB;
    for (int q = 0; q < RB; ++q)
      for (int k = 0; k < K; ++k) {
        double v = 0.0;
        if (q < rb) {
          const size_t o = (size_t)(g->row0 + r0 + q) * g->lda + k;
          v = g->dtype == 0 ? (double)orc_bf16_to_f32(((const uint16_t *)g->A)[o])
                            : (double)orc_e4m3_to_f32(((const uint8_t *)g->A)[o]) * g->scale_a;
        }
        a[(size_t)q * K + k] = v;
      }
    for (int c0 = 0; c0 < g->tn; c0 += CB) {
      const int cb = g->tn - c0 < CB ? g->tn - c0 : CB;
      double acc[RB][CB];
      for (int q = 0; q < RB; ++q)
        for (int c = 0; c < CB; ++c) acc[q][c] = 0.0;
      if (cb == CB) {
        for (int k = 0; k < K; ++k) {
          const double *b = g->bt + (size_t)k * g->tn + c0;
          const double a0 = a[k], a1 = a[K + k], a2 = a[2 * (size_t)K + k],
                       a3 = a[3 * (size_t)K + k];
          for (int c = 0; c < CB; ++c) {
            acc[0][c] += a0 * b[c];
            acc[1][c] += a1 * b[c];
            acc[2][c] += a2 * b[c];
            acc[3][c] += a3 * b[c];
          }
        }
      } else {
        for (int k = 0; k < K; ++k) {
          const double *b = g->bt + (size_t)k * g->tn + c0;
          for (int q = 0; q < RB; ++q)
            for (int c = 0; c < cb; ++c) acc[q][c] += a[(size_t)q * K + k] * b[c];
        }
      }
      for (int q = 0; q < rb; ++q)
        for (int c = 0; c < cb; ++c) g->out[(size_t)(r0 + q) * g->tn + c0 + c] = acc[q][c];
    }
  }
  free(a);
  return NULL;
}

/* Decodes B columns [col0, col0 + tn) into k-major doubles; thread `part`
 * of `parts` takes the k rows part, part + parts, ... */
typedef struct {
  const void *B;
  double *bt;
  int dtype, K, ldb, col0, tn, part, parts;
  double scale_b;
} decode_job;

static void *decode_worker(void *p) {
  const decode_job *d = (const decode_job *)p;
  for (int k = d->part; k < d->K; k += d->parts)
    for (int j = 0; j < d->tn; ++j) {
      const size_t o = (size_t)(d->col0 + j) * d->ldb + k;
      d->bt[(size_t)k * d->tn + j] =
          d->dtype == 0 ? (double)orc_bf16_to_f32(((const uint16_t *)d->B)[o])
                        : (double)orc_e4m3_to_f32(((const uint8_t *)d->B)[o]) * d->scale_b;
    }
  return NULL;
}

void orc_gemm_tiles_f64(const void *A, const void *B, int dtype, int K, int lda, int ldb,
                        int ntiles, const int *tiles, double scale_a, double scale_b,
                        double *out, int threads) {
  const int t = pick_threads(threads);
  const int nt = t < 256 ? t : 256;
  pthread_t th[256];
  decode_job dj[256];
  size_t off = 0;
  for (int i = 0; i < ntiles; ++i) {
    const int row0 = tiles[4 * i], col0 = tiles[4 * i + 1];
    const int tm = tiles[4 * i + 2], tn = tiles[4 * i + 3];
    double *bt = (double *)malloc(sizeof(double) * (size_t)K * tn);
    int started = 0;
    for (int k = 0; k < nt; ++k) {
      dj[k] = (decode_job){B, bt, dtype, K, ldb, col0, tn, k, nt, scale_b};
      if (pthread_create(&th[started], NULL, decode_worker, &dj[k]) == 0) ++started;
      else decode_worker(&dj[k]); /* no thread: decode this share here */
    }
    for (int k = 0; k < started; ++k) pthread_join(th[k], NULL);
    tiles_job g = {A, bt, out + off, dtype, K, lda, row0, tm, tn, scale_a, 0,
                   PTHREAD_MUTEX_INITIALIZER};
    started = 0;
    for (int k = 0; k < nt; ++k)
      if (pthread_create(&th[started], NULL, tiles_worker, &g) == 0) ++started;
    if (started == 0) tiles_worker(&g); /* every row block on this thread */
    for (int k = 0; k < started; ++k) pthread_join(th[k], NULL);
    pthread_mutex_destroy(&g.mu);
    free(bt);
    off += (size_t)tm * tn;
  }
}

typedef struct {
  const uint16_t *A, *B;
  float *C;
  int N, K, row0, rows, c_lo, c_hi;
} gemm_job;

/* One thread owns the output columns [c_lo, c_hi) of every sampled row, so
 * each B element is decoded once in total.  B is decoded in blocks of
 * KB x 64, stored k-major; the inner loop is an axpy over 64 output columns
 * for four rows at once (each output accumulates in k order, no sum is
 * reassociated).  Built for several ISA levels (ifunc dispatch at load time)
 * so the timed baseline uses the host's vector width without tying the build
 * to it. */
__attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))
static void *gemm_worker(void *p) {
  gemm_job *g = (gemm_job *)p;
  enum { KB = 256, CB = 64, RB = 4 };
  float *bt = (float *)malloc(sizeof(float) * KB * CB);
  float *a = (float *)malloc(sizeof(float) * KB * RB);
  for (int r = 0; r < g->rows; ++r)
    for (int c = g->c_lo; c < g->c_hi; ++c) g->C[(size_t)r * g->N + c] = 0.0f;
  for (int k0 = 0; k0 < g->K; k0 += KB) {
    const int kb = g->K - k0 < KB ? g->K - k0 : KB;
    for (int c0 = g->c_lo; c0 < g->c_hi; c0 += CB) {
      const int cb = g->c_hi - c0 < CB ? g->c_hi - c0 : CB;
      for (int c = 0; c < CB; ++c)
        for (int k = 0; k < kb; ++k)
          bt[k * CB + c] = c < cb ? bf16_to_f32(g->B[(size_t)(c0 + c) * g->K + k0 + k]) : 0.0f;
      for (int r0 = 0; r0 < g->rows; r0 += RB) {
        const int rb = g->rows - r0 < RB ? g->rows - r0 : RB;
        for (int q = 0; q < RB; ++q)
          for (int k = 0; k < kb; ++k)
            a[q * KB + k] = q < rb ? bf16_to_f32(g->A[(size_t)(g->row0 + r0 + q) * g->K + k0 + k])
                                   : 0.0f;
        float acc[RB][CB];
        for (int q = 0; q < RB; ++q)
          for (int c = 0; c < CB; ++c) acc[q][c] = 0.0f;
        for (int k = 0; k < kb; ++k) {
          const float *brow = bt + k * CB;
          const float a0 = a[k], a1 = a[KB + k], a2 = a[2 * KB + k], a3 = a[3 * KB + k];
          for (int c = 0; c < CB; ++c) {
            const float b = brow[c];
            acc[0][c] += a0 * b;
            acc[1][c] += a1 * b;
            acc[2][c] += a2 * b;
            acc[3][c] += a3 * b;
          }
        }
        for (int q = 0; q < rb; ++q) {
          float *crow = g->C + (size_t)(r0 + q) * g->N + c0;
          for (int c = 0; c < cb; ++c) crow[c] += acc[q][c];
        }
      }
    }
  }
  free(a);
  free(bt);
  return NULL;
}

void orc_gemm_bf16_rows_f32(const uint16_t *A, const uint16_t *B, float *C,
                            int N, int K, int row0, int rows, int threads) {
  int t = pick_threads(threads);
  const int blocks = (N + 63) / 64; /* column blocks of 64 */
  if (t > blocks) t = blocks > 0 ? blocks : 1;
  pthread_t th[256];
  gemm_job jobs[256];
  int used = 0;
  for (int k = 0; k < t; ++k) {
    int lo = (int)((long)blocks * k / t) * 64, hi = (int)((long)blocks * (k + 1) / t) * 64;
    if (hi > N) hi = N;
    if (lo >= hi) continue;
    jobs[used] = (gemm_job){A, B, C, N, K, row0, rows, lo, hi};
    pthread_create(&th[used], NULL, gemm_worker, &jobs[used]);
    ++used;
  }
  for (int k = 0; k < used; ++k) pthread_join(th[k], NULL);
}
