// stream.cu — HBM read and copy streams (reference src/mem_global.cu:13-26).
//
// Copy: persistent grid of k CTAs per SM, 256 threads each; every thread
// keeps UNROLL vectors of VB bytes in flight (VB = 16 or 32: sm_100 has
// 256-bit global loads/stores).  Each load instruction of a warp covers one
// contiguous 32 * VB byte span, loads use the non-coherent path without L1
// allocation and stores are evict-first, so nothing of the stream is kept.
//
// Sum: the same loop; each loaded vector is summed pairwise in fp32 and
// added to one of UNROLL fp64 accumulators per thread, which are combined
// per CTA in fp64; each CTA writes one fp64 partial to the workspace, and a
// one-CTA combine kernel, launched behind the sum with programmatic stream
// serialization (its launch overlaps the sum; it waits for the sum grid to
// complete), adds the partials in CTA order, so the result does not depend
// on CTA scheduling and nothing in the workspace needs clearing first.
#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

constexpr int kStreamThreads = 256;

template <int VB>
struct Vec;

template <>
struct Vec<16> {
  uint32_t w[4];
  __device__ __forceinline__ void load(const void *p) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "l"(p));
  }
  __device__ __forceinline__ void store(void *p) const {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3])
                 : "memory");
  }
  __device__ __forceinline__ float pairwise_sum() const {
    return (__uint_as_float(w[0]) + __uint_as_float(w[1])) +
           (__uint_as_float(w[2]) + __uint_as_float(w[3]));
  }
};

template <>
struct Vec<32> {
  uint32_t w[8];
  __device__ __forceinline__ void load(const void *p) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                   "=r"(w[6]), "=r"(w[7])
                 : "l"(p));
  }
  __device__ __forceinline__ void store(void *p) const {
    asm volatile("st.global.cs.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(w[0]),
                 "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
  }
  __device__ __forceinline__ float pairwise_sum() const {
    return ((__uint_as_float(w[0]) + __uint_as_float(w[1])) +
            (__uint_as_float(w[2]) + __uint_as_float(w[3]))) +
           ((__uint_as_float(w[4]) + __uint_as_float(w[5])) +
            (__uint_as_float(w[6]) + __uint_as_float(w[7])));
  }
};

// Copies nvec vectors of VB bytes, then the tail bytes [nvec*VB, bytes).
template <int VB, int UNROLL>
__global__ void __launch_bounds__(kStreamThreads) k_stream_copy(char *__restrict__ dst,
                                                                const char *__restrict__ src,
                                                                size_t nvec, size_t bytes) {
  const size_t tile = (size_t)kStreamThreads * UNROLL;
  const size_t step = (size_t)gridDim.x * tile;
  for (size_t base = blockIdx.x * tile; base < nvec; base += step) {
    if (base + tile <= nvec) {
      Vec<VB> v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        v[u].load(src + (base + (size_t)u * kStreamThreads + threadIdx.x) * VB);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        v[u].store(dst + (base + (size_t)u * kStreamThreads + threadIdx.x) * VB);
    } else {
#pragma unroll 1
      for (int u = 0; u < UNROLL; ++u) {
        size_t i = base + (size_t)u * kStreamThreads + threadIdx.x;
        if (i < nvec) {
          Vec<VB> v;
          v.load(src + i * VB);
          v.store(dst + i * VB);
        }
      }
    }
  }
  if (blockIdx.x == 0)
    for (size_t i = nvec * VB + threadIdx.x; i < bytes; i += kStreamThreads) dst[i] = src[i];
}

// Any alignment: byte-granular grid-stride copy.
__global__ void k_copy_bytes(char *__restrict__ dst, const char *__restrict__ src, size_t bytes) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < bytes;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

struct SumWorkspace {
  unsigned int reserved[64];  // header (256 bytes); keeps the partials on their own lines
  double partial[1];          // one per CTA
};

__device__ __forceinline__ double block_sum_f64(double v, double *smem) {
  v = dev::warp_sum_f64(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  double r = 0.0;
  if (warp == 0) {
    r = lane < (int)(blockDim.x >> 5) ? smem[lane] : 0.0;
    r = dev::warp_sum_f64(r);
  }
  __syncthreads();
  return r;  // valid in warp 0
}

// Sums src[0:n) into one fp64 partial per CTA.  `head` floats before the
// first 16-byte boundary and the tail after the last whole vector are added
// by CTA 0.  The kernel lets its dependent (k_sum_combine, launched with
// programmatic stream serialization) start at once; that kernel waits for
// this grid to finish before it reads the partials.
template <int VB, int UNROLL>
__global__ void __launch_bounds__(kStreamThreads) k_stream_sum(const float *__restrict__ src,
                                                               size_t n, size_t head,
                                                               SumWorkspace *ws) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int F = VB / 4;  // floats per vector
  const float *body = src + head;
  const size_t nvec = (n - head) / F;
  // Each vector's F floats are added pairwise in fp32 (error of a few ulp of
  // a value of order sqrt(F)); the vector sums accumulate in fp64.
  double acc[UNROLL];
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) acc[u] = 0.0;

  const size_t tile = (size_t)kStreamThreads * UNROLL;
  const size_t step = (size_t)gridDim.x * tile;
  for (size_t base = blockIdx.x * tile; base < nvec; base += step) {
    if (base + tile <= nvec) {
      Vec<VB> v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        v[u].load(body + (base + (size_t)u * kStreamThreads + threadIdx.x) * F);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) acc[u] += static_cast<double>(v[u].pairwise_sum());
    } else {
#pragma unroll 1
      for (int u = 0; u < UNROLL; ++u) {
        size_t i = base + (size_t)u * kStreamThreads + threadIdx.x;
        if (i < nvec) {
          Vec<VB> v;
          v.load(body + i * F);
          acc[0] += static_cast<double>(v.pairwise_sum());
        }
      }
    }
  }
  double t = 0.0;
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) t += acc[u];
  if (blockIdx.x == 0) {
    for (size_t i = threadIdx.x; i < head; i += kStreamThreads) t += src[i];
    for (size_t i = head + nvec * F + threadIdx.x; i < n; i += kStreamThreads) t += src[i];
  }
  __shared__ double red[kStreamThreads / 32];
  const double b = block_sum_f64(t, red);
  if (threadIdx.x == 0) ws->partial[blockIdx.x] = b;
}

// Fixed-order combine of the per-CTA partials (deterministic sums).  Its
// griddepcontrol.wait returns once the sum grid has completed and its
// writes are visible.
__global__ void __launch_bounds__(kStreamThreads) k_sum_combine(const SumWorkspace *ws,
                                                                int parts, double *out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double s = 0.0;
  for (int i = threadIdx.x; i < parts; i += kStreamThreads) s += ws->partial[i];
  __shared__ double red[kStreamThreads / 32];
  s = block_sum_f64(s, red);
  if (threadIdx.x == 0) *out = s;
}

struct CopyConfig {
  int vec_bytes, unroll, ctas_per_sm;
};

// Default launch shape of the copy stream.
constexpr CopyConfig kCopyDefault = {32, 2, 2};
constexpr int kSumVec = 32, kSumUnroll = 4, kSumCtasPerSm = 4;

int stream_grid(size_t units, size_t per_cta, int ctas_per_sm) {
  size_t want = (units + per_cta - 1) / per_cta;
  size_t cap = static_cast<size_t>(current_sm_count()) * ctas_per_sm;
  if (want > cap) want = cap;
  return want == 0 ? 1 : static_cast<int>(want);
}

template <int VB, int U>
void launch_copy(char *d, const char *s, size_t bytes, int ctas_per_sm, cudaStream_t st) {
  size_t nvec = bytes / VB;
  int grid = stream_grid(nvec, (size_t)kStreamThreads * U, ctas_per_sm);
  k_stream_copy<VB, U><<<grid, kStreamThreads, 0, st>>>(d, s, nvec, bytes);
}

int copy_impl(void *dst, const void *src, size_t bytes, CopyConfig cfg, cmb_stream_t stream) {
  if (bytes == 0) return CMB_OK;
  if (dst == nullptr || src == nullptr) return fail(CMB_ERR_INVALID_ARG, "stream copy: null pointer");
  char *d = static_cast<char *>(dst);
  const char *s = static_cast<const char *>(src);
  const uintptr_t mis = (reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s));
  if (cfg.ctas_per_sm < 1 || cfg.ctas_per_sm > 8)
    return fail(CMB_ERR_INVALID_ARG, "stream copy: ctas_per_sm %d not in [1, 8]", cfg.ctas_per_sm);
  if (cfg.vec_bytes == 32 && (mis & 31) != 0) cfg.vec_bytes = 16;
  if ((mis & 15) != 0) {
    int grid = stream_grid(bytes, kStreamThreads * 16, cfg.ctas_per_sm);
    k_copy_bytes<<<grid, kStreamThreads, 0, stream>>>(d, s, bytes);
    CMB_LAUNCH_CHECK();
    return CMB_OK;
  }
  const int u = cfg.unroll;
  if (cfg.vec_bytes == 16) {
    if (u == 1) launch_copy<16, 1>(d, s, bytes, cfg.ctas_per_sm, stream);
    else if (u == 2) launch_copy<16, 2>(d, s, bytes, cfg.ctas_per_sm, stream);
    else if (u == 4) launch_copy<16, 4>(d, s, bytes, cfg.ctas_per_sm, stream);
    else if (u == 8) launch_copy<16, 8>(d, s, bytes, cfg.ctas_per_sm, stream);
    else return fail(CMB_ERR_INVALID_ARG, "stream copy: unroll %d not in {1,2,4,8}", u);
  } else if (cfg.vec_bytes == 32) {
    if (u == 1) launch_copy<32, 1>(d, s, bytes, cfg.ctas_per_sm, stream);
    else if (u == 2) launch_copy<32, 2>(d, s, bytes, cfg.ctas_per_sm, stream);
    else if (u == 4) launch_copy<32, 4>(d, s, bytes, cfg.ctas_per_sm, stream);
    else if (u == 8) launch_copy<32, 8>(d, s, bytes, cfg.ctas_per_sm, stream);
    else return fail(CMB_ERR_INVALID_ARG, "stream copy: unroll %d not in {1,2,4,8}", u);
  } else {
    return fail(CMB_ERR_INVALID_ARG, "stream copy: vec_bytes %d not 16 or 32", cfg.vec_bytes);
  }
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

int sum_grid_cap() { return current_sm_count() * kSumCtasPerSm; }

}  // namespace

// Used by the no-allocation and host-buffer variants in other files.
int stream_sum_launch(const float *src, size_t n, double *out, void *ws, int max_grid,
                      cudaStream_t stream) {
  const size_t head = ((16 - (reinterpret_cast<uintptr_t>(src) & 15)) & 15) / 4;
  const size_t h = head < n ? head : n;
  const size_t nvec = (n - h) / (kSumVec / 4);
  int grid = stream_grid(nvec, (size_t)kStreamThreads * kSumUnroll, kSumCtasPerSm);
  if (grid > max_grid) grid = max_grid;
  SumWorkspace *w = static_cast<SumWorkspace *>(ws);
  if (((reinterpret_cast<uintptr_t>(src) + h * 4) & 31) == 0)
    k_stream_sum<32, kSumUnroll><<<grid, kStreamThreads, 0, stream>>>(src, n, h, w);
  else
    k_stream_sum<16, kSumUnroll><<<grid, kStreamThreads, 0, stream>>>(src, n, h, w);
  CMB_LAUNCH_CHECK();
  // The combine is launched behind the sum with programmatic stream
  // serialization, so its launch overlaps the sum instead of following it.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CMB_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_sum_combine, static_cast<const SumWorkspace *>(w), grid,
                                  out));
  return CMB_OK;
}

size_t stream_sum_workspace_for_grid(int grid) {
  return offsetof(SumWorkspace, partial) + sizeof(double) * static_cast<size_t>(grid);
}

}  // namespace cmb

using namespace cmb;

extern "C" int cmb_stream_copy(void *dst, const void *src, size_t bytes, cmb_stream_t stream) {
  return copy_impl(dst, src, bytes, kCopyDefault, stream);
}

extern "C" int cmb_stream_copy_tuned(void *dst, const void *src, size_t bytes, int vec_bytes,
                                     int unroll, int ctas_per_sm, cmb_stream_t stream) {
  return copy_impl(dst, src, bytes, CopyConfig{vec_bytes, unroll, ctas_per_sm}, stream);
}

extern "C" size_t cmb_stream_sum_workspace_bytes(size_t n) {
  (void)n;
  return stream_sum_workspace_for_grid(sum_grid_cap());
}

extern "C" int cmb_stream_sum_f32(const float *src, size_t n, double *out_sum, void *workspace,
                                  size_t workspace_bytes, cmb_stream_t stream) {
  if (out_sum == nullptr || workspace == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32: null out_sum or workspace");
  if (n > 0 && src == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32: null src");
  if ((reinterpret_cast<uintptr_t>(src) & 3) != 0)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32: src not 4-byte aligned");
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32: workspace not 16-byte aligned");
  const size_t need = cmb_stream_sum_workspace_bytes(n);
  if (workspace_bytes < need)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32: workspace %zu bytes < %zu needed",
                workspace_bytes, need);
  return stream_sum_launch(src, n, out_sum, workspace, sum_grid_cap(), stream);
}
