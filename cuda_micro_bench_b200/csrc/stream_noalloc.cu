// stream_noalloc.cu — the read-stream sum for callers that cannot allocate
// device memory.
//
// cmb_stream_sum_f32 needs a caller-allocated workspace (a 256-byte header
// and one fp64 partial per CTA).  Some callers cannot call cudaMalloc: code
// whose device memory is all owned by another allocator (a framework's
// caching allocator or a fixed arena), or latency-critical paths that cannot
// afford cudaMalloc/cudaFree, which may synchronise the device.  For them,
// cmb_stream_sum_f32_noalloc keeps that workspace in a file-scope device
// array of fixed size instead.  It runs the same kernel with the same launch
// shape, so its result equals cmb_stream_sum_f32's for the same input.
#include "cmb_device.cuh"
#include "cmb_host.h"

namespace cmb {

int stream_sum_launch(const float *src, size_t n, double *out, void *ws, int max_grid,
                      cudaStream_t stream);
size_t stream_sum_workspace_for_grid(int grid);

namespace {

// Room for 4096 per-CTA partials after the 256-byte header: 33,024 bytes,
// enough for the sum's grid (4 CTAs per SM) on GPUs of up to 1024 SMs.
constexpr int kNoAllocMaxCtas = 4096;
constexpr size_t kNoAllocScratchBytes = 256 + sizeof(double) * kNoAllocMaxCtas;

// One copy per GPU that loads the library, kept until the process exits.
// Every call on a device shares it.
static __device__ __align__(256) unsigned char g_sum_scratch[kNoAllocScratchBytes];

// Device address of g_sum_scratch in the current context.  In host code the
// symbol is only a stand-in; a kernel must be given this address.  It is
// looked up on every call rather than cached: after cudaDeviceReset() (or
// with another context current) the runtime loads the module again and the
// array can sit at a different address.  The lookup is a host-side table
// read once the module is loaded.
void *scratch_address_for_current_device(int *err) {
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_sum_scratch);
  if (e != cudaSuccess || p == nullptr) {
    *err = fail(CMB_ERR_CUDA, "cmb_stream_sum_f32_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(e));
    return nullptr;
  }
  return p;
}

}  // namespace
}  // namespace cmb

using namespace cmb;

extern "C" size_t cmb_stream_sum_noalloc_max_ctas(void) { return kNoAllocMaxCtas; }

extern "C" int cmb_stream_sum_f32_noalloc(const float *src, size_t n, double *out_sum,
                                          cmb_stream_t stream) {
  if (out_sum == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32_noalloc: null out_sum");
  if (n > 0 && src == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32_noalloc: null src");
  if ((reinterpret_cast<uintptr_t>(src) & 3) != 0)
    return fail(CMB_ERR_INVALID_ARG, "cmb_stream_sum_f32_noalloc: src not 4-byte aligned");
  // The sum launches one CTA per partial, up to the same cap as
  // cmb_stream_sum_f32 (whose workspace size encodes it).
  const size_t need = cmb_stream_sum_workspace_bytes(n);
  const size_t header = stream_sum_workspace_for_grid(0);
  const int max_grid = static_cast<int>((need - header) / sizeof(double));
  if (need > kNoAllocScratchBytes)
    return fail(CMB_ERR_INVALID_ARG,
                "cmb_stream_sum_f32_noalloc: this GPU's sum grid needs %d CTA partials (%zu "
                "bytes); the static scratch holds %d (%zu bytes)",
                max_grid, need, kNoAllocMaxCtas, kNoAllocScratchBytes);
  int err = CMB_OK;
  void *scratch = scratch_address_for_current_device(&err);
  if (scratch == nullptr) return err;
  // The partials are written before they are read, so nothing needs zeroing.
  return stream_sum_launch(src, n, out_sum, scratch, max_grid, stream);
}
