// stream_host.cpp — host-buffer stream copy: the copy probe as a caller with
// data in host memory sees it (host -> device, device copy, device -> host),
// with consecutive chunks overlapped on three streams so the two PCIe
// directions and the HBM copy run at the same time.
#include <mutex>
#include <vector>

#include "cmb_host.h"

namespace cmb {
namespace {

constexpr int kMaxSlots = 8;

struct HostCopyStreams {
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  cudaEvent_t in_ready[kMaxSlots], out_ready[kMaxSlots], in_free[kMaxSlots], out_free[kMaxSlots];
  bool ok = false;
};

std::mutex g_copy_mu;
HostCopyStreams g_copy_per_dev[64];

HostCopyStreams *streams_for_current_device() {
  std::mutex &mu = g_copy_mu;
  HostCopyStreams *per_dev = g_copy_per_dev;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  HostCopyStreams &s = per_dev[dev];
  if (!s.ok) {
    if (cudaStreamCreateWithFlags(&s.h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s.comp, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s.d2h, cudaStreamNonBlocking) != cudaSuccess)
      return nullptr;
    for (int i = 0; i < kMaxSlots; ++i) {
      if (cudaEventCreateWithFlags(&s.in_ready[i], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&s.out_ready[i], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&s.in_free[i], cudaEventDisableTiming) != cudaSuccess ||
          cudaEventCreateWithFlags(&s.out_free[i], cudaEventDisableTiming) != cudaSuccess)
        return nullptr;
    }
    s.ok = true;
  }
  return &s;
}

}  // namespace

// Destroys the staging streams and events of device `dev` (before a device
// reset, which would leave their handles dangling).
void host_copy_release_streams(int dev) {
  if (dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lock(g_copy_mu);
  HostCopyStreams &s = g_copy_per_dev[dev];
  if (!s.ok) return;
  cudaStreamDestroy(s.h2d);
  cudaStreamDestroy(s.comp);
  cudaStreamDestroy(s.d2h);
  for (int i = 0; i < kMaxSlots; ++i) {
    cudaEventDestroy(s.in_ready[i]);
    cudaEventDestroy(s.out_ready[i]);
    cudaEventDestroy(s.in_free[i]);
    cudaEventDestroy(s.out_free[i]);
  }
  s = HostCopyStreams{};
}

}  // namespace cmb

using namespace cmb;

extern "C" int cmb_stream_copy_host(void *host_dst, const void *host_src, size_t bytes,
                                    void *dev_a, void *dev_b, size_t dev_bytes, size_t chunk) {
  if (bytes == 0) return CMB_OK;
  if (!host_dst || !host_src || !dev_a || !dev_b)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_copy_host: null pointer");
  if (chunk == 0 || dev_bytes < 2 * chunk)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_copy_host: need dev_bytes >= 2*chunk > 0");
  HostCopyStreams *s = streams_for_current_device();
  if (!s) return fail(CMB_ERR_CUDA, "cmb_stream_copy_host: stream/event creation failed");
  int slots = static_cast<int>(dev_bytes / chunk);
  if (slots > kMaxSlots) slots = kMaxSlots;
  char *a = static_cast<char *>(dev_a), *b = static_cast<char *>(dev_b);
  const char *hs = static_cast<const char *>(host_src);
  char *hd = static_cast<char *>(host_dst);
  const size_t nchunks = (bytes + chunk - 1) / chunk;
  const auto enqueue = [&]() -> int {
    for (size_t c = 0; c < nchunks; ++c) {
      const int k = static_cast<int>(c % slots);
      const size_t off = c * chunk, len = off + chunk <= bytes ? chunk : bytes - off;
      if (c >= (size_t)slots) CMB_CUDA_TRY(cudaStreamWaitEvent(s->h2d, s->in_free[k], 0));
      CMB_CUDA_TRY(cudaMemcpyAsync(a + k * chunk, hs + off, len, cudaMemcpyHostToDevice, s->h2d));
      CMB_CUDA_TRY(cudaEventRecord(s->in_ready[k], s->h2d));
      CMB_CUDA_TRY(cudaStreamWaitEvent(s->comp, s->in_ready[k], 0));
      if (c >= (size_t)slots) CMB_CUDA_TRY(cudaStreamWaitEvent(s->comp, s->out_free[k], 0));
      int rc = cmb_stream_copy(b + k * chunk, a + k * chunk, len, s->comp);
      if (rc != CMB_OK) return rc;
      CMB_CUDA_TRY(cudaEventRecord(s->in_free[k], s->comp));
      CMB_CUDA_TRY(cudaEventRecord(s->out_ready[k], s->comp));
      CMB_CUDA_TRY(cudaStreamWaitEvent(s->d2h, s->out_ready[k], 0));
      CMB_CUDA_TRY(cudaMemcpyAsync(hd + off, b + k * chunk, len, cudaMemcpyDeviceToHost, s->d2h));
      CMB_CUDA_TRY(cudaEventRecord(s->out_free[k], s->d2h));
    }
    return CMB_OK;
  };
  const int rc = enqueue();
  // Wait for everything enqueued, on success and on failure alike, so the
  // caller's host buffers are no longer in use when this returns.
  const cudaError_t e1 = cudaStreamSynchronize(s->d2h), e2 = cudaStreamSynchronize(s->comp),
                    e3 = cudaStreamSynchronize(s->h2d);
  if (rc != CMB_OK) return rc;
  for (cudaError_t e : {e1, e2, e3})
    if (e != cudaSuccess)
      return fail(CMB_ERR_CUDA, "cmb_stream_copy_host: cudaStreamSynchronize: %s",
                  cudaGetErrorString(e));
  return CMB_OK;
}
