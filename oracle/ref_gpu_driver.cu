// Driver around the reference's own probe kernels and sections, compiled for
// sm_100a from the reference sources in place by oracle/Makefile (target
// `ref-gpu`).  Test infrastructure, run on a B200 to
//   fixtures  pin the oracle: the reference kernels' outputs on small inputs
//             (hash fill, pointer-chase endpoint on a given link array,
//             stream copy, constant-operand mma.sync sums), written as JSON;
//   sections  record the reference's own probe numbers on B200
//             (benchmark_global_memory, _cache, _tma, _tensor_core_extended)
//             in its results.json format, for comparison with this build.
// Usage: ref_gpu fixtures <links.bin> <out.json> | ref_gpu sections <out.json>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "bench_common.h"
#include "memory_chase.h"
#include "result_logger.h"

namespace cmb {
// Kernels and sections the reference defines in its .cu files.
__global__ void kernel_stream_copy(const uint4 *src, uint4 *dst, int n);
__global__ void kernel_hmma_bf16_throughput(float *out, int iters);
__global__ void kernel_hmma_int8_throughput(int *out, int iters);
void benchmark_global_memory();
void benchmark_cache();
void benchmark_tma();
void benchmark_tensor_core_extended();
}  // namespace cmb

#define CK(x)                                                                          \
  do {                                                                                 \
    cudaError_t e_ = (x);                                                              \
    if (e_ != cudaSuccess) {                                                           \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
      exit(2);                                                                         \
    }                                                                                  \
  } while (0)

static int fixtures(const char *links_path, const char *out_path) {
  using namespace cmb;
  FILE *out = fopen(out_path, "w");
  if (!out) return 2;
  fprintf(out, "{\n");
  // 1. kernel_init_stream on 4099 words
  {
    const int n = 4099;
    unsigned int *d;
    CK(cudaMalloc(&d, n * 4));
    kernel_init_stream<<<4, 256>>>(d, n);
    CK(cudaGetLastError());
    std::vector<unsigned int> h(n);
    CK(cudaMemcpy(h.data(), d, n * 4, cudaMemcpyDeviceToHost));
    fprintf(out, "  \"init_stream_4099\": [");
    for (int i = 0; i < n; ++i) fprintf(out, "%s%u", i ? "," : "", h[i]);
    fprintf(out, "],\n");
    CK(cudaFree(d));
  }
  // 2. kernel_random_chase_cg on the given link array
  {
    FILE *f = fopen(links_path, "rb");
    if (!f) return 2;
    std::vector<unsigned int> links;
    unsigned int w;
    while (fread(&w, 4, 1, f) == 1) links.push_back(w);
    fclose(f);
    unsigned int *d;
    unsigned long long *o;
    CK(cudaMalloc(&d, links.size() * 4));
    CK(cudaMalloc(&o, 16));
    CK(cudaMemcpy(d, links.data(), links.size() * 4, cudaMemcpyHostToDevice));
    const int cases[3][2] = {{0, 1}, {7, 1000}, {1024, 4096 * 3 + 5}};
    fprintf(out, "  \"chase_cg\": [");
    for (int c = 0; c < 3; ++c) {
      kernel_random_chase_cg<<<1, 1>>>(d, cases[c][0], cases[c][1], o);
      CK(cudaGetLastError());
      unsigned long long h[2];
      CK(cudaMemcpy(h, o, 16, cudaMemcpyDeviceToHost));
      fprintf(out, "%s{\"warmup\": %d, \"iters\": %d, \"final\": %llu}", c ? ", " : "", cases[c][0],
              cases[c][1], h[1]);
    }
    fprintf(out, "],\n");
    CK(cudaFree(d));
    CK(cudaFree(o));
  }
  // 3. kernel_stream_copy of 1 MiB of init_stream data: identity
  {
    const int nvec = (1 << 20) / 16;
    uint4 *a, *b;
    CK(cudaMalloc(&a, nvec * 16));
    CK(cudaMalloc(&b, nvec * 16));
    kernel_init_stream<<<64, 256>>>(reinterpret_cast<unsigned int *>(a), nvec * 4);
    kernel_stream_copy<<<64, 256>>>(a, b, nvec);
    CK(cudaGetLastError());
    std::vector<unsigned int> ha(nvec * 4), hb(nvec * 4);
    CK(cudaMemcpy(ha.data(), a, nvec * 16, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(hb.data(), b, nvec * 16, cudaMemcpyDeviceToHost));
    fprintf(out, "  \"stream_copy_1mib_identical\": %s,\n",
            memcmp(ha.data(), hb.data(), nvec * 16) == 0 ? "true" : "false");
    CK(cudaFree(a));
    CK(cudaFree(b));
  }
  // 4. constant-operand mma.sync sums (one warp, `iters` MMAs)
  {
    const int iters = 1000;
    float *f;
    int *i;
    CK(cudaMalloc(&f, 32 * 4));
    CK(cudaMalloc(&i, 32 * 4));
    kernel_hmma_bf16_throughput<<<1, 32>>>(f, iters);
    kernel_hmma_int8_throughput<<<1, 32>>>(i, iters);
    CK(cudaGetLastError());
    float hf[32];
    int hi[32];
    CK(cudaMemcpy(hf, f, sizeof(hf), cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(hi, i, sizeof(hi), cudaMemcpyDeviceToHost));
    fprintf(out, "  \"hmma_bf16_sum_iters1000\": %.1f,\n  \"hmma_int8_sum_iters1000\": %d\n", hf[0],
            hi[0]);
    CK(cudaFree(f));
    CK(cudaFree(i));
  }
  fprintf(out, "}\n");
  fclose(out);
  return 0;
}

int main(int argc, char **argv) {
  if (argc == 4 && strcmp(argv[1], "fixtures") == 0) return fixtures(argv[2], argv[3]);
  if (argc == 3 && strcmp(argv[1], "sections") == 0) {
    cmb::benchmark_global_memory();
    cmb::benchmark_cache();
    cmb::benchmark_tma();
    cmb::benchmark_tensor_core_extended();
    cmb::g_results.writeJson(argv[2]);
    return 0;
  }
  fprintf(stderr, "usage: %s fixtures <links.bin> <out.json> | sections <out.json>\n", argv[0]);
  return 2;
}
