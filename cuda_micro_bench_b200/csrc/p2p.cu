// p2p.cu — multi-GPU probe: NVLink peer copies (new; the reference only asks
// cudaDeviceCanAccessPeer, src/pcie.cu:100-112).
//
// Two ways to move bytes to another GPU over NVLink / NVSwitch:
//   - in-kernel peer stores: SMs of the sending GPU load their own HBM with
//     wide vector loads and issue 16-byte stores to a pointer that maps the
//     receiver's memory (cudaIpcOpenMemHandle in multi-process use,
//     cudaDeviceEnablePeerAccess in one process);
//   - the copy engines: cudaMemcpyAsync between the two devices' pointers.
// A "job" is one (src, dst, bytes) copy; a scatter runs up to 8 jobs at once
// (one per destination GPU), which covers the ring (one job) and the
// all-to-all (one job per peer).  No TMA and no collective library is used,
// and no kernel waits on another GPU: completion is observed on the host.
#include <cstring>
#include <mutex>

#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {
namespace {

constexpr int kMaxJobs = 8;
constexpr int kP2PThreads = 256;

struct Jobs {
  const char *src[kMaxJobs];
  char *dst[kMaxJobs];
  size_t bytes[kMaxJobs];
};

// blockIdx.y = job; the CTAs of a job stride over its tiles of 256 threads
// x 4 16-byte vectors: each thread keeps four loads of its own HBM in
// flight, and each warp store instruction writes 512 contiguous bytes of the
// destination.
__global__ void __launch_bounds__(kP2PThreads) k_p2p_store(Jobs jobs) {
  constexpr int kUnroll = 4;
  const int j = blockIdx.y;
  const uint4 *__restrict__ src = reinterpret_cast<const uint4 *>(jobs.src[j]);
  uint4 *__restrict__ dst = reinterpret_cast<uint4 *>(jobs.dst[j]);
  const size_t bytes = jobs.bytes[j];
  const size_t nvec = bytes / 16;
  const size_t tile = (size_t)kP2PThreads * kUnroll;
  for (size_t base = blockIdx.x * tile; base < nvec; base += (size_t)gridDim.x * tile) {
    if (base + tile <= nvec) {
      uint4 v[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) v[k] = __ldg(src + base + k * kP2PThreads + threadIdx.x);
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) dst[base + k * kP2PThreads + threadIdx.x] = v[k];
    } else {
      for (int k = 0; k < kUnroll; ++k) {
        const size_t i = base + k * kP2PThreads + threadIdx.x;
        if (i < nvec) dst[i] = __ldg(src + i);
      }
    }
  }
  if (blockIdx.x == 0) {
    const char *s8 = jobs.src[j];
    char *d8 = jobs.dst[j];
    for (size_t i = nvec * 16 + threadIdx.x; i < bytes; i += kP2PThreads) d8[i] = s8[i];
  }
}

struct CeStreams {
  cudaStream_t s[kMaxJobs] = {};
  cudaEvent_t fork = nullptr, join[kMaxJobs] = {};
  bool ok = false;
};

CeStreams *ce_streams_for_current_device() {
  static std::mutex mu;
  static CeStreams per_dev[64];
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

extern "C" int cmb_p2p_scatter_store(void *const *dst, const void *const *src, const size_t *bytes,
                                     int n, int ctas_per_job, cmb_stream_t stream) {
  int rc = check_jobs("cmb_p2p_scatter_store", dst, src, bytes, n);
  if (rc) return rc;
  Jobs jobs = {};
  size_t most = 0;
  for (int j = 0; j < n; ++j) {
    if ((reinterpret_cast<uintptr_t>(dst[j]) | reinterpret_cast<uintptr_t>(src[j])) & 15)
      return fail(CMB_ERR_INVALID_ARG, "cmb_p2p_scatter_store: job %d not 16-byte aligned", j);
    jobs.src[j] = static_cast<const char *>(src[j]);
    jobs.dst[j] = static_cast<char *>(dst[j]);
    jobs.bytes[j] = bytes[j];
    most = bytes[j] > most ? bytes[j] : most;
  }
  if (most == 0) return CMB_OK;
  if (ctas_per_job <= 0) ctas_per_job = (current_sm_count() * 2 + n - 1) / n;
  size_t want = (most / 16 + kP2PThreads * 4 - 1) / (kP2PThreads * 4);
  if ((size_t)ctas_per_job > want) ctas_per_job = static_cast<int>(want == 0 ? 1 : want);
  k_p2p_store<<<dim3(ctas_per_job, n), kP2PThreads, 0, stream>>>(jobs);
  CMB_LAUNCH_CHECK();
  return CMB_OK;
}

extern "C" int cmb_p2p_scatter_copy_engine(void *const *dst, const void *const *src,
                                           const size_t *bytes, int n, cmb_stream_t stream) {
  int rc = check_jobs("cmb_p2p_scatter_copy_engine", dst, src, bytes, n);
  if (rc) return rc;
  CeStreams *c = ce_streams_for_current_device();
  if (c == nullptr) return fail(CMB_ERR_CUDA, "copy-engine streams could not be created");
  // fork the jobs onto one stream each, so every destination's copy engine
  // work runs concurrently, then join them back into `stream`
  CMB_CUDA_TRY(cudaEventRecord(c->fork, stream));
  for (int j = 0; j < n; ++j) {
    CMB_CUDA_TRY(cudaStreamWaitEvent(c->s[j], c->fork, 0));
    if (bytes[j] > 0)
      CMB_CUDA_TRY(cudaMemcpyAsync(dst[j], src[j], bytes[j], cudaMemcpyDefault, c->s[j]));
    CMB_CUDA_TRY(cudaEventRecord(c->join[j], c->s[j]));
    CMB_CUDA_TRY(cudaStreamWaitEvent(stream, c->join[j], 0));
  }
  return CMB_OK;
}
