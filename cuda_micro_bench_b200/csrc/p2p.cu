// p2p.cu — multi-GPU probe: NVLink peer copies (new; the reference only asks
// cudaDeviceCanAccessPeer, src/pcie.cu:100-112).
//
// Three ways to move bytes to another GPU over NVLink / NVSwitch:
//   - in-kernel peer stores: SMs of the sending GPU load their own HBM with
//     wide vector loads and issue 16- or 32-byte stores to a pointer that
//     maps the receiver's memory (cudaIpcOpenMemHandle in multi-process use,
//     cudaDeviceEnablePeerAccess in one process);
//   - in-kernel bulk copies: one thread per CTA streams chunks of its own
//     HBM into a shared-memory ring with cp.async.bulk loads (this GPU's
//     memory only, one destination CTA) and writes each chunk to the peer
//     pointer with one cp.async.bulk store;
//   - the copy engines: cudaMemcpyAsync between the two devices' pointers.
// A "job" is one (src, dst, bytes) copy; a scatter runs up to 8 jobs at once
// (one per destination GPU), which covers the ring (one job) and the
// all-to-all (one job per peer).  No collective library is used, and no
// kernel waits on another GPU: completion is observed on the host.
#include <cstring>
#include <mutex>
#include <type_traits>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

constexpr int kMaxJobs = 8;
constexpr int kP2PThreads = 256;
constexpr int kBulkCtasPerJob = 32;  // default CTAs per job of a bulk scatter

struct Jobs {
  const char *src[kMaxJobs];
  char *dst[kMaxJobs];
  size_t bytes[kMaxJobs];
};

// 32-byte vector of the store kernel.
struct V32 {
  uint32_t w[8];
};

__device__ __forceinline__ V32 ld_v32(const void *p) {
  V32 v;
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]),
                 "=r"(v.w[5]), "=r"(v.w[6]), "=r"(v.w[7])
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v32(void *p, const V32 &v) {
  asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]),
               "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]),
               "r"(v.w[7])
               : "memory");
}

// blockIdx.y = job; the CTAs of a job stride over its tiles of 256 threads
// x 4 vectors of VB bytes (16 or 32): each thread keeps four loads of its own
// HBM in flight, and each warp store instruction writes 32 * VB contiguous
// bytes of the destination.
template <int VB>
__global__ void __launch_bounds__(kP2PThreads) k_p2p_store(Jobs jobs) {
  constexpr int kUnroll = 4;
  using V = typename std::conditional<VB == 16, uint4, V32>::type;
  const int j = blockIdx.y;
  const char *__restrict__ src = jobs.src[j];
  char *__restrict__ dst = jobs.dst[j];
  const size_t bytes = jobs.bytes[j];
  const size_t nvec = bytes / VB;
  const size_t tile = (size_t)kP2PThreads * kUnroll;
  for (size_t base = blockIdx.x * tile; base < nvec; base += (size_t)gridDim.x * tile) {
    if (base + tile <= nvec) {
      V v[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const size_t i = base + k * kP2PThreads + threadIdx.x;
        if constexpr (VB == 16) v[k] = __ldg(reinterpret_cast<const uint4 *>(src) + i);
        else v[k] = ld_v32(src + i * 32);
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const size_t i = base + k * kP2PThreads + threadIdx.x;
        if constexpr (VB == 16) reinterpret_cast<uint4 *>(dst)[i] = v[k];
        else st_v32(dst + i * 32, v[k]);
      }
    } else {
      for (int k = 0; k < kUnroll; ++k) {
        const size_t i = base + k * kP2PThreads + threadIdx.x;
        if (i < nvec) {
          if constexpr (VB == 16)
            reinterpret_cast<uint4 *>(dst)[i] = __ldg(reinterpret_cast<const uint4 *>(src) + i);
          else
            st_v32(dst + i * 32, ld_v32(src + i * 32));
        }
      }
    }
  }
  if (blockIdx.x == 0)
    for (size_t i = nvec * VB + threadIdx.x; i < bytes; i += kP2PThreads) dst[i] = src[i];
}

// Bulk-copy form: blockIdx.y = job; CTA x takes chunks x, x + gridDim.x, ...
// of the job's 16-byte-aligned body.  One thread keeps S - G + 1 chunk loads
// and G chunk stores in flight over an S-stage ring: after the store of
// chunk i it waits until at most G - 1 stores still read shared memory, then
// reloads the stage of chunk i + 1 - G with chunk i + 1 - G + S.  The body's
// last (< 16) bytes are copied by plain stores in CTA 0.
template <int S, int G>
__global__ void __launch_bounds__(32) k_p2p_bulk(Jobs jobs, uint32_t chunk, int *status) {
  static_assert(G >= 1 && 2 * G <= S, "stores in flight must leave loads in flight");
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full[S];
  const int j = blockIdx.y;
  const char *__restrict__ src = jobs.src[j];
  char *__restrict__ dst = jobs.dst[j];
  const size_t bytes = jobs.bytes[j];
  const size_t body = bytes & ~static_cast<size_t>(15);
  const size_t nchunks = (body + chunk - 1) / chunk;
  const size_t mine =
      nchunks > blockIdx.x ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (threadIdx.x == 0 && mine > 0) {
    for (int s = 0; s < S; ++s) dev::mbar_init(dev::smem_addr(&full[s]), 1);
    dev::fence_mbar_init();
    const auto off = [&](size_t i) { return (blockIdx.x + i * gridDim.x) * (size_t)chunk; };
    const auto len = [&](size_t i) {
      const size_t o = off(i);
      return static_cast<uint32_t>(body - o < chunk ? body - o : chunk);
    };
    size_t issued = 0;  // chunks whose load has been issued
    const auto load = [&](size_t i) {
      const int s = static_cast<int>(i % S);
      const uint32_t bar = dev::smem_addr(&full[s]);
      dev::mbar_arrive_expect_tx(bar, len(i));
      dev::bulk_load(dev::smem_addr(ring + (size_t)s * chunk), src + off(i), len(i), bar);
      issued = i + 1;
    };
    for (size_t i = 0; i < mine && i < (size_t)S; ++i) load(i);
    for (size_t i = 0; i < mine; ++i) {
      const int s = static_cast<int>(i % S);
      if (!dev::mbar_wait_bounded(dev::smem_addr(&full[s]), static_cast<uint32_t>(i / S) & 1)) {
        dev::report_status(status, CMB_ERR_TIMEOUT);
        // wait (bounded) for the loads still writing the ring before the
        // CTA's shared memory goes away
        for (size_t k = i; k < issued; ++k)
          if (!dev::mbar_wait_bounded(dev::smem_addr(&full[k % S]),
                                      static_cast<uint32_t>(k / S) & 1, 100000000ull))
            break;
        break;
      }
      dev::bulk_store(dst + off(i), dev::smem_addr(ring + (size_t)s * chunk), len(i));
      dev::bulk_commit_group();
      if (i + 1 >= (size_t)G && i + 1 - G + S < mine) {
        dev::bulk_wait_group_read<G - 1>();
        load(i + 1 - G + S);
      }
    }
    dev::bulk_wait_group<0>();  // every store has written its bytes
  }
  if (blockIdx.x == 0)
    for (size_t i = body + threadIdx.x; i < bytes; i += 32) dst[i] = src[i];
}

struct CeStreams {
  cudaStream_t s[kMaxJobs] = {};
  cudaEvent_t fork = nullptr, join[kMaxJobs] = {};
  bool ok = false;
};

std::mutex g_ce_mu;
CeStreams g_ce_per_dev[64];

CeStreams *ce_streams_for_current_device() {
  std::mutex &mu = g_ce_mu;
  CeStreams *per_dev = g_ce_per_dev;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  CeStreams &c = per_dev[dev];
  if (!c.ok) {
    if (cudaEventCreateWithFlags(&c.fork, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    for (int i = 0; i < kMaxJobs; ++i)
      if (cudaStreamCreateWithFlags(&c.s[i], cudaStreamNonBlocking) != cudaSuccess ||
          cudaEventCreateWithFlags(&c.join[i], cudaEventDisableTiming) != cudaSuccess)
        return nullptr;
    c.ok = true;
  }
  return &c;
}

int check_jobs(const char *fn, void *const *dst, const void *const *src, const size_t *bytes,
               int n) {
  if (n < 1 || n > kMaxJobs) return fail(CMB_ERR_INVALID_ARG, "%s: %d jobs not in [1, 8]", fn, n);
  if (dst == nullptr || src == nullptr || bytes == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "%s: null job arrays", fn);
  for (int j = 0; j < n; ++j) {
    if (bytes[j] > 0 && (dst[j] == nullptr || src[j] == nullptr))
      return fail(CMB_ERR_INVALID_ARG, "%s: job %d has a null pointer", fn, j);
  }
  return CMB_OK;
}

}  // namespace

// Destroys the copy-engine streams and events of device `dev` (before a
// device reset, which would leave their handles dangling).
void p2p_release_streams(int dev) {
  if (dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lock(g_ce_mu);
  CeStreams &c = g_ce_per_dev[dev];
  if (!c.ok) return;
  for (int i = 0; i < kMaxJobs; ++i) {
    cudaStreamDestroy(c.s[i]);
    cudaEventDestroy(c.join[i]);
  }
  cudaEventDestroy(c.fork);
  c = CeStreams{};
}

}  // namespace cmb

using namespace cmb;

extern "C" int cmb_p2p_alloc(size_t bytes, void **out) {
  if (out == nullptr || bytes == 0) return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_alloc: bad arguments");
  CMB_CUDA_TRY(cudaMalloc(out, bytes));
  return CMB_OK;
}

extern "C" int cmb_p2p_free(void *ptr) {
  if (ptr != nullptr) CMB_CUDA_TRY(cudaFree(ptr));
  return CMB_OK;
}

extern "C" size_t cmb_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int cmb_ipc_get_handle(void *base, void *handle_out) {
  if (base == nullptr || handle_out == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  CMB_CUDA_TRY(cudaIpcGetMemHandle(&h, base));
  memcpy(handle_out, &h, sizeof(h));
  return CMB_OK;
}

extern "C" int cmb_ipc_open(const void *handle, void **peer_ptr) {
  if (handle == nullptr || peer_ptr == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  CMB_CUDA_TRY(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return CMB_OK;
}

extern "C" int cmb_ipc_close(void *peer_ptr) {
  if (peer_ptr != nullptr) CMB_CUDA_TRY(cudaIpcCloseMemHandle(peer_ptr));
  return CMB_OK;
}

extern "C" int cmb_p2p_enable_peer(int peer_device) {
  int can = 0, dev = 0;
  CMB_CUDA_TRY(cudaGetDevice(&dev));
  CMB_CUDA_TRY(cudaDeviceCanAccessPeer(&can, dev, peer_device));
  if (!can)
    return fail(CMB_ERR_UNSUPPORTED, "device %d cannot access device %d's memory", dev, peer_device);
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return CMB_OK;
  }
  if (e != cudaSuccess)
    return fail(CMB_ERR_CUDA, "cudaDeviceEnablePeerAccess(%d): %s", peer_device,
                cudaGetErrorString(e));
  return CMB_OK;
}

namespace cmb {
namespace {

int scatter_store(void *const *dst, const void *const *src, const size_t *bytes, int n,
                  int ctas_per_job, int vec_bytes, cudaStream_t stream) {
  int rc = check_jobs("cmb_p2p_scatter_store", dst, src, bytes, n);
  if (rc) return rc;
  if (vec_bytes != 16 && vec_bytes != 32)
    return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_store: vec_bytes %d not 16 or 32", vec_bytes);
  Jobs jobs = {};
  size_t most = 0;
  for (int j = 0; j < n; ++j) {
    if ((reinterpret_cast<uintptr_t>(dst[j]) | reinterpret_cast<uintptr_t>(src[j])) & (vec_bytes - 1))
      return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_store: job %d not %d-byte aligned", j,
                  vec_bytes);
    jobs.src[j] = static_cast<const char *>(src[j]);
    jobs.dst[j] = static_cast<char *>(dst[j]);
    jobs.bytes[j] = bytes[j];
    most = bytes[j] > most ? bytes[j] : most;
  }
  if (most == 0) return CMB_OK;
  if (ctas_per_job <= 0) ctas_per_job = (current_sm_count() * 2 + n - 1) / n;
  const size_t tile = (size_t)kP2PThreads * 4 * vec_bytes;
  size_t want = (most + tile - 1) / tile;
  if ((size_t)ctas_per_job > want) ctas_per_job = static_cast<int>(want == 0 ? 1 : want);
  if (vec_bytes == 16) k_p2p_store<16><<<dim3(ctas_per_job, n), kP2PThreads, 0, stream>>>(jobs);
  else k_p2p_store<32><<<dim3(ctas_per_job, n), kP2PThreads, 0, stream>>>(jobs);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

}  // namespace
}  // namespace cmb

extern "C" int cmb_p2p_scatter_store(void *const *dst, const void *const *src, const size_t *bytes,
                                     int n, int ctas_per_job, cmb_stream_t stream) {
  // 32-byte vectors when every job allows them
  int vb = 32;
  for (int j = 0; j < n && j < kMaxJobs; ++j)
    if (dst != nullptr && src != nullptr &&
        ((reinterpret_cast<uintptr_t>(dst[j]) | reinterpret_cast<uintptr_t>(src[j])) & 31))
      vb = 16;
  return scatter_store(dst, src, bytes, n, ctas_per_job, vb, stream);
}

extern "C" int cmb_p2p_scatter_store_tuned(void *const *dst, const void *const *src,
                                           const size_t *bytes, int n, int ctas_per_job,
                                           int vec_bytes, cmb_stream_t stream) {
  return scatter_store(dst, src, bytes, n, ctas_per_job, vec_bytes, stream);
}

namespace cmb {
namespace {

template <int S, int G>
int launch_bulk(const Jobs &jobs, int n, int ctas_per_job, uint32_t chunk, int *status,
                cudaStream_t stream) {
  const size_t smem = (size_t)S * chunk;
  auto kern = k_p2p_bulk<S, G>;
  CMB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  kern<<<dim3(ctas_per_job, n), 32, smem, stream>>>(jobs, chunk, status);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

int scatter_bulk(void *const *dst, const void *const *src, const size_t *bytes, int n,
                 int ctas_per_job, int chunk_bytes, int stages, int *status, cudaStream_t stream) {
  const char *fn = "cmb_p2p_scatter_bulk";
  int rc = check_jobs(fn, dst, src, bytes, n);
  if (rc) return rc;
  if (chunk_bytes == 0) chunk_bytes = 16 << 10;
  if (stages == 0) stages = 8;
  if (chunk_bytes < 16 || chunk_bytes % 16 != 0 || chunk_bytes > (64 << 10))
    return fail(CMB_ERR_INVALID_ARG, "%s: chunk_bytes %d not a multiple of 16 in [16, 65536]", fn,
                chunk_bytes);
  if (stages != 4 && stages != 8)
    return fail(CMB_ERR_INVALID_ARG, "%s: stages %d not 4 or 8", fn, stages);
  if ((size_t)stages * chunk_bytes > (size_t)(227 << 10))
    return fail(CMB_ERR_INVALID_ARG, "%s: %d stages x %d bytes exceed 227 KiB of shared memory",
                fn, stages, chunk_bytes);
  Jobs jobs = {};
  size_t most = 0;
  for (int j = 0; j < n; ++j) {
    if ((reinterpret_cast<uintptr_t>(dst[j]) | reinterpret_cast<uintptr_t>(src[j])) & 15)
      return fail(CMB_ERR_INVALID_ARG, "%s: job %d not 16-byte aligned", fn, j);
    jobs.src[j] = static_cast<const char *>(src[j]);
    jobs.dst[j] = static_cast<char *>(dst[j]);
    jobs.bytes[j] = bytes[j];
    most = bytes[j] > most ? bytes[j] : most;
  }
  if (most == 0) return CMB_OK;
  // 32 CTAs per job (at most one per SM in all): on a ring they reach the
  // SM-side write ceiling (~680 GB/s per GPU on B200 NVLink 5, the same as
  // peer stores from every SM) and leave the rest of the GPU free.
  if (ctas_per_job <= 0) {
    const int per_sm = current_sm_count() / n;
    ctas_per_job = per_sm < kBulkCtasPerJob ? (per_sm < 1 ? 1 : per_sm) : kBulkCtasPerJob;
  }
  const size_t want = (most + chunk_bytes - 1) / chunk_bytes;
  if ((size_t)ctas_per_job > want) ctas_per_job = static_cast<int>(want == 0 ? 1 : want);
  const uint32_t c = static_cast<uint32_t>(chunk_bytes);
  return stages == 4 ? launch_bulk<4, 2>(jobs, n, ctas_per_job, c, status, stream)
                     : launch_bulk<8, 4>(jobs, n, ctas_per_job, c, status, stream);
}

}  // namespace
}  // namespace cmb

extern "C" int cmb_p2p_scatter_bulk(void *const *dst, const void *const *src, const size_t *bytes,
                                    int n, int ctas_per_job, int *status, cmb_stream_t stream) {
  return scatter_bulk(dst, src, bytes, n, ctas_per_job, 0, 0, status, stream);
}

extern "C" int cmb_p2p_scatter_bulk_tuned(void *const *dst, const void *const *src,
                                          const size_t *bytes, int n, int ctas_per_job,
                                          int chunk_bytes, int stages, int *status,
                                          cmb_stream_t stream) {
  return scatter_bulk(dst, src, bytes, n, ctas_per_job, chunk_bytes, stages, status, stream);
}

namespace cmb {
namespace {

int scatter_copy_engine(void *const *dst, const void *const *src, const size_t *bytes, int n,
                        int streams, cmb_stream_t stream) {
  int rc = check_jobs("cmb_p2p_scatter_copy_engine", dst, src, bytes, n);
  if (rc) return rc;
  if (streams < 1 || streams > kMaxJobs)
    return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_copy_engine: %d streams not in [1, 8]",
                streams);
  CeStreams *c = ce_streams_for_current_device();
  if (c == nullptr) return fail(CMB_ERR_CUDA, "copy-engine streams could not be created");
  // Fork onto `streams` internal streams, job j on stream j % streams in the
  // given order (jobs that share a stream run one after another), then join
  // them back into `stream`.
  const int used = streams < n ? streams : n;
  CMB_CUDA_TRY(cudaEventRecord(c->fork, stream));
  for (int q = 0; q < used; ++q) CMB_CUDA_TRY(cudaStreamWaitEvent(c->s[q], c->fork, 0));
  for (int j = 0; j < n; ++j)
    if (bytes[j] > 0)
      CMB_CUDA_TRY(cudaMemcpyAsync(dst[j], src[j], bytes[j], cudaMemcpyDefault, c->s[j % used]));
  for (int q = 0; q < used; ++q) {
    CMB_CUDA_TRY(cudaEventRecord(c->join[q], c->s[q]));
    CMB_CUDA_TRY(cudaStreamWaitEvent(stream, c->join[q], 0));
  }
  return CMB_OK;
}

}  // namespace
}  // namespace cmb

namespace cmb {
namespace {

// Job j's first head_bytes(j) go by the copy engines, the rest by peer
// stores from the SMs; the split falls on a 4 KiB boundary so both parts
// keep the job's alignment.
size_t hybrid_head(size_t bytes, int ce_permille) {
  const size_t head = bytes / 1000 * static_cast<size_t>(ce_permille) +
                      bytes % 1000 * static_cast<size_t>(ce_permille) / 1000;
  return head / 4096 * 4096;
}

int scatter_hybrid(void *const *dst, const void *const *src, const size_t *bytes, int n,
                   int ce_permille, int ce_streams, cmb_stream_t stream) {
  int rc = check_jobs("cmb_p2p_scatter_hybrid", dst, src, bytes, n);
  if (rc) return rc;
  if (ce_permille < 0 || ce_permille > 1000)
    return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_hybrid: ce_permille %d not in [0, 1000]",
                ce_permille);
  if (ce_streams < 1 || ce_streams > kMaxJobs)
    return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_hybrid: %d streams not in [1, 8]",
                ce_streams);
  void *tail_dst[kMaxJobs];
  const void *tail_src[kMaxJobs];
  size_t head[kMaxJobs], tail[kMaxJobs];
  int vb = 32;
  for (int j = 0; j < n; ++j) {
    if ((reinterpret_cast<uintptr_t>(dst[j]) | reinterpret_cast<uintptr_t>(src[j])) & 15)
      return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_hybrid: job %d not 16-byte aligned", j);
    head[j] = hybrid_head(bytes[j], ce_permille);
    tail[j] = bytes[j] - head[j];
    tail_dst[j] = static_cast<char *>(dst[j]) + head[j];
    tail_src[j] = static_cast<const char *>(src[j]) + head[j];
    if ((reinterpret_cast<uintptr_t>(dst[j]) | reinterpret_cast<uintptr_t>(src[j])) & 31) vb = 16;
  }
  CeStreams *c = ce_streams_for_current_device();
  if (c == nullptr) return fail(CMB_ERR_CUDA, "copy-engine streams could not be created");
  // heads: forked onto the copy-engine streams, job j on stream j % ce_streams
  const int used = ce_streams < n ? ce_streams : n;
  CMB_CUDA_TRY(cudaEventRecord(c->fork, stream));
  for (int q = 0; q < used; ++q) CMB_CUDA_TRY(cudaStreamWaitEvent(c->s[q], c->fork, 0));
  for (int j = 0; j < n; ++j)
    if (head[j] > 0)
      CMB_CUDA_TRY(cudaMemcpyAsync(dst[j], src[j], head[j], cudaMemcpyDefault, c->s[j % used]));
  // tails: peer stores on `stream`, meanwhile
  rc = scatter_store(tail_dst, tail_src, tail, n, 0, vb, stream);
  // join the heads back into `stream` (also after a failed launch, so the
  // internal streams are never left ahead of it)
  for (int q = 0; q < used; ++q) {
    CMB_CUDA_TRY(cudaEventRecord(c->join[q], c->s[q]));
    CMB_CUDA_TRY(cudaStreamWaitEvent(stream, c->join[q], 0));
  }
  return rc;
}

}  // namespace
}  // namespace cmb

extern "C" int cmb_p2p_scatter_hybrid(void *const *dst, const void *const *src,
                                      const size_t *bytes, int n, int ce_permille, int ce_streams,
                                      cmb_stream_t stream) {
  return scatter_hybrid(dst, src, bytes, n, ce_permille, ce_streams, stream);
}

extern "C" int cmb_p2p_scatter_copy_engine(void *const *dst, const void *const *src,
                                           const size_t *bytes, int n, cmb_stream_t stream) {
  return scatter_copy_engine(dst, src, bytes, n, n, stream);
}

extern "C" int cmb_p2p_scatter_copy_engine_tuned(void *const *dst, const void *const *src,
                                                 const size_t *bytes, int n, int streams,
                                                 cmb_stream_t stream) {
  return scatter_copy_engine(dst, src, bytes, n, streams, stream);
}
