// sections.cpp — the probe sections (see sections.h) and the CLI.
#include "sections.h"

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../../include/cmb_b200.h"
#include "../cmb_host.h"
#include "result_logger.h"

namespace cmb {
namespace {

#define TRY(expr)                   \
  do {                              \
    const int rc_ = (expr);         \
    if (rc_ != CMB_OK) return rc_;  \
  } while (0)

constexpr uint64_t kStreamSeed = 0x5EED, kChaseSeed = 0xC0DA, kGemmSeed = 0x6E33;

// Device buffer owned by a section (each section frees what it allocates,
// as the reference's sections do).
struct DevBuf {
  void *p = nullptr;
  DevBuf() = default;
  DevBuf(const DevBuf &) = delete;
  ~DevBuf() {
    if (p != nullptr) cudaFree(p);
  }
  int alloc(size_t bytes) {
    CMB_CUDA_TRY(cudaMalloc(&p, bytes == 0 ? 1 : bytes));
    return CMB_OK;
  }
  template <class T>
  T *as() const {
    return static_cast<T *>(p);
  }
};

// Milliseconds of each of `runs` launches of fn (CUDA events on the legacy
// default stream); returns the median after dropping the first `drop`
// (src/mem_global.cu:42-53 drops one of six and takes the median of five).
// A pair of timing events, destroyed on every return path.
struct EventPair {
  cudaEvent_t a = nullptr, b = nullptr;
  EventPair() = default;
  EventPair(const EventPair &) = delete;
  ~EventPair() {
    if (a != nullptr) cudaEventDestroy(a);
    if (b != nullptr) cudaEventDestroy(b);
  }
  int create() {
    CMB_CUDA_TRY(cudaEventCreate(&a));
    CMB_CUDA_TRY(cudaEventCreate(&b));
    return CMB_OK;
  }
};

template <class F>
int time_median(F fn, int runs, int drop, double *ms_out) {
  EventPair ev;
  TRY(ev.create());
  std::vector<double> ms;
  for (int r = 0; r < runs; ++r) {
    CMB_CUDA_TRY(cudaEventRecord(ev.a, nullptr));
    TRY(fn());
    CMB_CUDA_TRY(cudaEventRecord(ev.b, nullptr));
    CMB_CUDA_TRY(cudaEventSynchronize(ev.b));
    float t = 0.f;
    CMB_CUDA_TRY(cudaEventElapsedTime(&t, ev.a, ev.b));
    if (r >= drop) ms.push_back(t);
  }
  if (ms.empty()) return fail(CMB_ERR_INVALID_ARG, "time_median: %d runs, %d dropped", runs, drop);
  std::sort(ms.begin(), ms.end());
  *ms_out = ms[ms.size() / 2];
  return CMB_OK;
}

double gib_per_s(double bytes, double ms) { return bytes / (ms * 1e-3) / (1024.0 * 1024.0 * 1024.0); }
double gb_per_s(double bytes, double ms) { return bytes / (ms * 1e-3) / 1e9; }
double nominal_ns(double cycles, int clock_khz) { return cycles * 1e6 / clock_khz; }

unsigned host_threads() {
  unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 1 : std::min(n, 64u);
}

// fp64 sum of the uniform stream cmb_fill_uniform_f32 writes (the same
// SplitMix64 formula, regenerated on the host).
double host_uniform_sum(size_t n, uint64_t seed) {
  const unsigned nt = host_threads();
  std::vector<double> part(nt, 0.0);
  std::vector<std::thread> pool;
  for (unsigned t = 0; t < nt; ++t)
    pool.emplace_back([&, t] {
      double s = 0.0;
      for (size_t i = n * t / nt; i < n * (t + 1) / nt; ++i) {
        uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        s += static_cast<double>(static_cast<float>(static_cast<uint32_t>(z >> 40)) * 0x1p-23f - 1.0f);
      }
      part[t] = s;
    });
  for (auto &th : pool) th.join();
  double s = 0.0;
  for (double v : part) s += v;
  return s;
}

double seconds_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// The host side of the stream probes, on the same data: the fp32 values the
// device summed and copied, summed in fp64 and copied by every host thread
// (contiguous block per thread).  `sum` must equal the fp64 reference sum of
// the seeded stream (same values, same order per block).
struct HostStream {
  double sum, sum_gbps, memcpy_gbps;
};

HostStream host_stream(const std::vector<float> &x) {
  const unsigned nt = host_threads();
  const size_t n = x.size();
  std::vector<float> y(n);
  std::vector<double> part(nt, 0.0);
  HostStream r{};
  {
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < nt; ++t)
      pool.emplace_back([&, t] {
        double s = 0.0;
        for (size_t i = n * t / nt; i < n * (t + 1) / nt; ++i) s += static_cast<double>(x[i]);
        part[t] = s;
      });
    for (auto &th : pool) th.join();
    r.sum_gbps = 4.0 * n / seconds_since(t0) / 1e9;
  }
  r.sum = 0.0;
  for (double v : part) r.sum += v;
  {
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < nt; ++t)
      pool.emplace_back([&, t] {
        const size_t a = n * t / nt, b = n * (t + 1) / nt;
        std::memcpy(y.data() + a, x.data() + a, (b - a) * sizeof(float));
      });
    for (auto &th : pool) th.join();
    r.memcpy_gbps = 2.0 * 4.0 * n / seconds_since(t0) / 1e9;
  }
  if (std::memcmp(x.data(), y.data(), n * sizeof(float)) != 0) r.memcpy_gbps = -1.0;
  return r;
}

int expect_equal(const void *a, const void *b, size_t bytes, bool *equal) {
  DevBuf cnt;
  TRY(cnt.alloc(sizeof(unsigned long long)));
  TRY(cmb_compare_bytes(a, b, bytes, cnt.as<unsigned long long>(), nullptr));
  unsigned long long h = 1;
  CMB_CUDA_TRY(cudaMemcpy(&h, cnt.p, sizeof(h), cudaMemcpyDeviceToHost));
  *equal = (h == 0);
  return CMB_OK;
}

// ------------------------------------------------------------ chase

struct ChaseResult {
  double cycles_per_hop, ns_per_hop;
  double host_ns_per_hop;  // the host walk of the same cycle (one thread)
};

// Dependent-load chase over `bytes` (include/memory_chase.h:11-59): the link
// array is built on the host, the endpoint is checked against a host walk
// (failure = CMB_ERR_MISMATCH), median of five samples.
int measure_chase(size_t bytes, bool bypass_l1, bool resident, ChaseResult *res) {
  const size_t words = bytes / 4, slots = bytes / 128;
  std::vector<uint32_t> links(words);
  TRY(cmb_chase_build_links(links.data(), bytes, kChaseSeed));
  // resident: warm the cycle twice, then 2^17 timed hops (the reference's
  // cache probes); cold: 1024 warm-up hops, then 2^24 hops (4 walks of the
  // 512 MiB cycle, the DRAM configuration).
  const uint64_t warmup = resident ? 2 * slots : 1024;
  const uint64_t hops = resident ? (1u << 17) : (1u << 24);
  uint32_t expect = 0;
  const auto walk0 = std::chrono::steady_clock::now();
  TRY(cmb_chase_host_walk(links.data(), words, warmup + hops, &expect));
  res->host_ns_per_hop = seconds_since(walk0) * 1e9 / static_cast<double>(warmup + hops);
  DevBuf d, out;
  TRY(d.alloc(bytes));
  TRY(out.alloc(4 * sizeof(uint64_t)));
  CMB_CUDA_TRY(cudaMemcpy(d.p, links.data(), bytes, cudaMemcpyHostToDevice));
  std::vector<double> cyc, ns;
  for (int s = 0; s < 5; ++s) {
    TRY(cmb_chase_run(d.as<uint32_t>(), words, warmup, hops, bypass_l1 ? 1 : 0, out.as<uint64_t>(),
                      nullptr));
    uint64_t h[4];
    CMB_CUDA_TRY(cudaMemcpy(h, out.p, sizeof(h), cudaMemcpyDeviceToHost));
    if (h[3] != 0) return fail(CMB_ERR_INVALID_ARG, "pointer chase: link array rejected");
    if (h[1] != expect)
      return fail(CMB_ERR_MISMATCH, "Pointer chase result mismatch (%llu != %u)",
                  static_cast<unsigned long long>(h[1]), expect);
    cyc.push_back(static_cast<double>(h[0]) / hops);
    ns.push_back(static_cast<double>(h[2]) / hops);
  }
  std::sort(cyc.begin(), cyc.end());
  std::sort(ns.begin(), ns.end());
  res->cycles_per_hop = cyc[2];
  res->ns_per_hop = ns[2];
  return CMB_OK;
}

// ------------------------------------------------------------ GEMM check

float bf16_bits_to_float(uint16_t v) {
  uint32_t u = static_cast<uint32_t>(v) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

float e4m3_to_float(uint8_t v) {
  __nv_fp8_e4m3 x;
  x.__x = v;
  return static_cast<float>(x);
}

// Runs fn(i) for i in [0, n) on all host threads.
template <class F>
void parallel_for(int n, F fn) {
  const int t = std::max(1, std::min<int>(n, static_cast<int>(std::thread::hardware_concurrency())));
  std::vector<std::thread> pool;
  std::atomic<int> next{0};
  for (int k = 0; k < t; ++k)
    pool.emplace_back([&] {
      for (int i = next++; i < n; i = next++) fn(i);
    });
  for (auto &th : pool) th.join();
}

// Max over `tiles` sampled T x T output tiles (the first and the last
// corner tile, then tiles drawn from a fixed LCG) of
// max|C - C_fp64| / max|C_fp64| within the tile: the max-norm reading of
// the stated "rel tol 1e-2".  Each fp64 product is summed in k order; the
// tile's B columns are decoded once (k-major) and the row blocks are spread
// over the host's threads.
template <bool kFp8>
double sampled_gemm_error(const std::vector<uint8_t> &A, const std::vector<uint8_t> &B,
                          const std::vector<float> &C, int M, int N, int K, double sa, double sb,
                          int tiles) {
  constexpr int T = 256, RB = 4, CB = 16;
  auto elem = [&](const std::vector<uint8_t> &X, size_t i, double s) -> double {
    if (kFp8) return e4m3_to_float(X[i]) * s;
    uint16_t v;
    std::memcpy(&v, &X[2 * i], 2);
    return bf16_bits_to_float(v);
  };
  double worst = 0.0;
  uint64_t r = 12345;
  std::vector<double> bt((size_t)K * T), ref((size_t)T * T);
  for (int t = 0; t < tiles; ++t) {
    r = r * 6364136223846793005ull + 1442695040888963407ull;
    int r0 = static_cast<int>((r >> 33) % (M / T)) * T;
    int c0 = static_cast<int>((r >> 13) % (N / T)) * T;
    if (t == 0) r0 = c0 = 0;
    if (t == 1) r0 = M - T, c0 = N - T;
    parallel_for(K, [&](int k) {
      for (int j = 0; j < T; ++j) bt[(size_t)k * T + j] = elem(B, (size_t)(c0 + j) * K + k, sb);
    });
    parallel_for(T / RB, [&](int blk) {
      std::vector<double> a((size_t)RB * K);
      for (int q = 0; q < RB; ++q)
        for (int k = 0; k < K; ++k) a[(size_t)q * K + k] = elem(A, (size_t)(r0 + blk * RB + q) * K + k, sa);
      for (int j0 = 0; j0 < T; j0 += CB) {
        double acc[RB][CB] = {};
        for (int k = 0; k < K; ++k) {
          const double *b = &bt[(size_t)k * T + j0];
          for (int q = 0; q < RB; ++q) {
            const double aq = a[(size_t)q * K + k];
            for (int j = 0; j < CB; ++j) acc[q][j] += aq * b[j];
          }
        }
        for (int q = 0; q < RB; ++q)
          for (int j = 0; j < CB; ++j) ref[(size_t)(blk * RB + q) * T + j0 + j] = acc[q][j];
      }
    });
    double ref_max = 0.0, err_max = 0.0;
    for (int i = 0; i < T; ++i)
      for (int j = 0; j < T; ++j) {
        const double s = ref[(size_t)i * T + j];
        const double c = C[(size_t)(r0 + i) * N + c0 + j];
        ref_max = std::max(ref_max, std::fabs(s));
        err_max = std::max(err_max, std::isfinite(c) ? std::fabs(c - s) : HUGE_VAL);
      }
    worst = std::max(worst, err_max / std::max(ref_max, 1e-300));
  }
  return worst;
}

}  // namespace

int query_device(int dev, DeviceInfo *info) {
  CMB_CUDA_TRY(cudaSetDevice(dev));
  cudaDeviceProp prop;
  CMB_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
  info->id = dev;
  info->name = prop.name;
  info->cc_major = prop.major;
  info->cc_minor = prop.minor;
  info->sm_count = prop.multiProcessorCount;
  info->max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
  info->max_warps_per_sm = prop.maxThreadsPerMultiProcessor / prop.warpSize;
  CMB_CUDA_TRY(cudaDeviceGetAttribute(&info->clock_rate_khz, cudaDevAttrClockRate, dev));
  CMB_CUDA_TRY(cudaDeviceGetAttribute(&info->memory_clock_khz, cudaDevAttrMemoryClockRate, dev));
  info->mem_bus_width = prop.memoryBusWidth;
  info->l2_cache_size = prop.l2CacheSize;
  info->total_global_mem = prop.totalGlobalMem;
  info->shared_mem_per_block_optin = prop.sharedMemPerBlockOptin;
  g_results.setDevice(info->name, std::to_string(info->cc_major) + "." + std::to_string(info->cc_minor),
                      info->sm_count, info->clock_rate_khz, info->memory_clock_khz,
                      info->mem_bus_width);
  return CMB_OK;
}

// --device: the device header and derived peaks (src/device_info.cu:6-59).
int section_device_info() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== Device Info ===\n  %s, cc %d.%d, %d SMs, %.2f GiB, L2 %d KiB, clock %.3f GHz\n",
         info.name.c_str(), info.cc_major, info.cc_minor, info.sm_count,
         info.total_global_mem / 1073741824.0, info.l2_cache_size / 1024,
         info.clock_rate_khz / 1e6);
  const double fp32 = (double)info.sm_count * 128 * 2 * info.clock_rate_khz / 1e9;
  const double mem_bw = (double)info.memory_clock_khz * 2 * info.mem_bus_width / 8.0 / 1e6;
  g_results.log("topology", "sm_count", info.sm_count, "");
  g_results.log("topology", "max_warps_per_sm", info.max_warps_per_sm, "");
  g_results.log("topology", "max_threads_per_sm", info.max_threads_per_sm, "");
  g_results.log("topology", "l2_cache_size_mb", info.l2_cache_size / (1024.0 * 1024.0), "MiB");
  g_results.log("topology", "shared_memory_per_block_optin_kb",
                info.shared_mem_per_block_optin / 1024.0, "KiB");
  g_results.log("clock", "core_clock_mhz", info.clock_rate_khz / 1000.0, "MHz");
  g_results.log("clock", "memory_clock_mhz", info.memory_clock_khz / 1000.0, "MHz");
  g_results.log("peak", "fp32_tflops", fp32, "TFLOP/s");
  g_results.log("peak", "memory_bw_theoretical_gbps", mem_bw, "GB/s");
  return CMB_OK;
}

int section_global_memory() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== Global Memory Benchmarks (median of 5) ===\n");
  const size_t sizes[] = {16ull << 20, 64ull << 20, 256ull << 20, 1ull << 30};
  double read_gib = 0, copy_gib = 0, read_gbs = 0, copy_gbs = 0, rel_err = 0;
  size_t reported = 0;
  bool copy_ok = true;
  for (size_t bytes : sizes) {
    if (bytes > info.total_global_mem / 4) continue;
    const size_t n = bytes / 4;
    DevBuf a, b, sum, ws;
    const size_t ws_bytes = cmb_stream_sum_workspace_bytes(n);
    TRY(a.alloc(bytes));
    TRY(b.alloc(bytes));
    TRY(sum.alloc(sizeof(double)));
    TRY(ws.alloc(ws_bytes));
    TRY(cmb_fill_uniform_f32(a.as<float>(), n, kStreamSeed, nullptr));
    double cms = 0, rms = 0;
    TRY(time_median([&] { return cmb_stream_copy(b.p, a.p, bytes, nullptr); }, 6, 1, &cms));
    bool eq = false;
    TRY(expect_equal(a.p, b.p, bytes, &eq));
    copy_ok = copy_ok && eq;
    TRY(time_median(
        [&] {
          return cmb_stream_sum_f32(a.as<float>(), n, sum.as<double>(), ws.p, ws_bytes, nullptr);
        },
        6, 1, &rms));
    double got = 0;
    CMB_CUDA_TRY(cudaMemcpy(&got, sum.p, sizeof(got), cudaMemcpyDeviceToHost));
    const double ref = host_uniform_sum(n, kStreamSeed);
    rel_err = std::fabs(got - ref) / std::max(std::fabs(ref), 1e-300);
    if (bytes == sizes[3]) {  // the host reference on the same 1 GiB
      std::vector<float> hx(n);
      CMB_CUDA_TRY(cudaMemcpy(hx.data(), a.p, bytes, cudaMemcpyDeviceToHost));
      const HostStream hs = host_stream(hx);
      if (hs.memcpy_gbps < 0) return fail(CMB_ERR_MISMATCH, "host reference memcpy differs");
      if (hs.sum != ref)
        return fail(CMB_ERR_MISMATCH, "host sum of the device stream %.17g != %.17g", hs.sum, ref);
      printf("  host reference (%u threads, 1 GiB): fp64 sum %.1f GB/s, memcpy %.1f GB/s "
             "(read+write)\n", host_threads(), hs.sum_gbps, hs.memcpy_gbps);
      g_results.log("host_ref", "cores", host_threads(), "threads");
      g_results.log("host_ref", "sum_gbps", hs.sum_gbps, "GB/s");
      g_results.log("host_ref", "memcpy_gbps", hs.memcpy_gbps, "GB/s");
    }
    copy_gib = gib_per_s(2.0 * bytes, cms);
    read_gib = gib_per_s((double)bytes, rms);
    copy_gbs = gb_per_s(2.0 * bytes, cms);
    read_gbs = gb_per_s((double)bytes, rms);
    reported = bytes;
    printf("  %5zu MiB: copy %.2f GiB/s (read+write, %s), read %.2f GiB/s (sum rel err %.1e)\n",
           bytes >> 20, copy_gib, eq ? "bit-exact" : "MISMATCH", read_gib, rel_err);
    if (!eq) return fail(CMB_ERR_MISMATCH, "stream copy output differs from its input");
    if (rel_err > 1e-5) return fail(CMB_ERR_MISMATCH, "stream sum rel err %.3g > 1e-5", rel_err);
  }
  g_results.log("memory_dram", "read_bw_gibps", read_gib, "GiB/s");
  g_results.log("memory_dram", "copy_max_bw_gibps", copy_gib, "GiB/s");
  g_results.log("memory", "dram_read_bw_gbps", read_gib * 1.073741824, "GB/s");
  g_results.log("memory_dram", "stream_working_set_bytes", (double)reported, "bytes");
  g_results.log("memory_dram", "copy_bw_gbps", copy_gbs, "GB/s");
  g_results.log("memory_dram", "copy_frac_of_8tbs_spec", copy_gbs / 8000.0, "");
  g_results.log("memory_dram", "read_frac_of_8tbs_spec", read_gbs / 8000.0, "");
  g_results.log("memory_dram", "copy_verified", copy_ok ? 1.0 : 0.0, "bool");
  g_results.log("memory_dram", "read_sum_rel_err", rel_err, "");
  g_results.log("memory_dram", "stream_seed", static_cast<double>(kStreamSeed), "seed");

  // DRAM latency: 512 MiB link array (well above the 126 MB L2), .cg loads.
  const size_t bytes = std::min<size_t>(512ull << 20, info.total_global_mem / 8);
  ChaseResult cr;
  TRY(measure_chase(bytes, true, false, &cr));
  const double ns = nominal_ns(cr.cycles_per_hop, info.clock_rate_khz);
  printf("  DRAM random chase (.cg, %zu MiB, 2^24 hops): %.2f cycles (%.2f nominal ns, %.2f ns "
         "measured)\n", bytes >> 20, cr.cycles_per_hop, ns, cr.ns_per_hop);
  g_results.log("memory", "dram_latency_cyc", cr.cycles_per_hop, "cycles");
  g_results.log("memory_dram", "pointer_chase_latency_ns", ns, "nominal ns");
  g_results.log("memory_dram", "pointer_chase_latency_ns_measured", cr.ns_per_hop, "ns");
  g_results.log("memory_dram", "chase_working_set_bytes", (double)bytes, "bytes");
  g_results.log("memory_dram", "chase_loads_per_sample", (double)(1u << 24), "loads");
  g_results.log("memory_dram", "chase_min_sector_footprint_bytes", (double)(bytes / 4), "bytes");
  g_results.log("memory_dram", "chase_endpoint_verified", 1.0, "bool");
  g_results.log("memory_dram", "chase_seed", static_cast<double>(kChaseSeed), "seed");
  printf("  host walk of the same cycle (one thread): %.2f ns per hop\n", cr.host_ns_per_hop);
  g_results.log("host_ref", "chase_ns_per_hop", cr.host_ns_per_hop, "ns");
  return CMB_OK;
}

int section_cache() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== Cache Benchmarks (random dependent loads, median of 5) ===\n");
  for (int kb = 4; kb <= 256; kb *= 2) {
    ChaseResult cr;
    TRY(measure_chase((size_t)kb * 1024, false, true, &cr));
    printf("    %4d KiB -> %.2f cycles/access\n", kb, cr.cycles_per_hop);
    char key[64];
    snprintf(key, sizeof(key), "l1_chase_%d_kb_cycles", kb);
    g_results.log("memory_cache", key, cr.cycles_per_hop, "cycles/access");
    if (kb == 4) g_results.log("memory", "l1_latency_cyc", cr.cycles_per_hop, "cycles");
  }
  const size_t l2_bytes = std::min<size_t>(8ull << 20, (size_t)info.l2_cache_size / 4);
  if (l2_bytes >= (1ull << 20)) {
    ChaseResult cr;
    TRY(measure_chase(l2_bytes, true, true, &cr));
    printf("  L2 (.cg, %zu KiB): %.2f cycles/access\n", l2_bytes / 1024, cr.cycles_per_hop);
    g_results.log("memory", "l2_latency_cyc", cr.cycles_per_hop, "cycles");
    g_results.log("memory_cache", "l2_chase_working_set_bytes", (double)l2_bytes, "bytes");
  }
  return CMB_OK;
}

// --memory-more: L2 aggregate read bandwidth (src/memory_more.cu:201-234):
// an L2-resident buffer of min(8 MiB, L2/4) read 1024 times by 4 CTAs per
// SM; median of five after one warm-up; the exact word sum is checked.
int section_memory_more() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== Memory (L2 aggregate bandwidth) ===\n");
  // 8 MiB (a multiple of the bulk path's 8 KiB chunks) stays in L2.
  const size_t bytes = std::min<size_t>(8ull << 20, (size_t)info.l2_cache_size / 4) & ~size_t(8191);
  const int passes = 1024;
  DevBuf buf, sum, st;
  TRY(buf.alloc(bytes));
  TRY(sum.alloc(sizeof(unsigned long long)));
  TRY(st.alloc(sizeof(int)));
  TRY(cmb_fill_hash_u32(buf.as<uint32_t>(), bytes / 4, nullptr));
  unsigned long long words = 0;
  for (size_t i = 0; i < bytes / 4; ++i) {
    uint32_t x = static_cast<uint32_t>(i) + 0x9e3779b9u;
    x = (x ^ (x >> 16)) * 0x85ebca6bu;
    x = (x ^ (x >> 13)) * 0xc2b2ae35u;
    words += x ^ (x >> 16);
  }
  // register loads (the reference's form) and bulk copies into shared memory
  double ms_ldg = 0, ms_bulk = 0;
  unsigned long long got = 0;
  TRY(time_median([&] { return cmb_l2_read(buf.p, bytes, passes, 0, sum.as<unsigned long long>(), nullptr); },
                  6, 1, &ms_ldg));
  CMB_CUDA_TRY(cudaMemcpy(&got, sum.p, sizeof(got), cudaMemcpyDeviceToHost));
  if (got != words * passes)
    return fail(CMB_ERR_MISMATCH, "L2 read: word sum %llu != %llu", got, words * passes);
  TRY(time_median([&] {
        return cmb_l2_read_bulk(buf.p, bytes, passes, sum.as<unsigned long long>(), st.as<int>(), nullptr);
      },
      6, 1, &ms_bulk));
  int status = 0;
  CMB_CUDA_TRY(cudaMemcpy(&got, sum.p, sizeof(got), cudaMemcpyDeviceToHost));
  CMB_CUDA_TRY(cudaMemcpy(&status, st.p, sizeof(status), cudaMemcpyDeviceToHost));
  if (status != 0) return fail(status, "L2 bulk read: a bounded wait expired");
  if (got != words * passes)
    return fail(CMB_ERR_MISMATCH, "L2 bulk read: word sum %llu != %llu", got, words * passes);
  const double total = (double)bytes * passes;
  const double ms = std::min(ms_ldg, ms_bulk);
  printf("  L2 aggregate BW (%zu KiB resident): .cg 16-byte register loads %.1f GB/s, bulk "
         "copies into shared memory %.1f GB/s\n",
         bytes >> 10, gb_per_s(total, ms_ldg), gb_per_s(total, ms_bulk));
  // the report's key carries the faster of the two reads of the same bytes
  g_results.log("memory_more", "l2_aggregate_bw_gibps", gib_per_s(total, ms), "GiB/s");
  g_results.log("memory_more", "l2_aggregate_bw_gbps", gb_per_s(total, ms), "GB/s");
  g_results.log("memory_more", "l2_aggregate_ldg_bw_gbps", gb_per_s(total, ms_ldg), "GB/s");
  g_results.log("memory_more", "l2_aggregate_bulk_bw_gbps", gb_per_s(total, ms_bulk), "GB/s");
  g_results.log("memory_more", "l2_aggregate_working_set_bytes", (double)bytes, "bytes");
  g_results.log("memory_more", "l2_aggregate_verified", 1.0, "bool");
  return CMB_OK;
}

// --pcie: pinned host <-> device copy bandwidth (src/pcie.cu:55-97): 64 MiB,
// ten copies per direction after a warm-up, device-timed.
// Pinned host buffer owned by a section.
struct PinnedBuf {
  void *p = nullptr;
  PinnedBuf() = default;
  PinnedBuf(const PinnedBuf &) = delete;
  ~PinnedBuf() {
    if (p != nullptr) cudaFreeHost(p);
  }
  int alloc(size_t bytes) {
    CMB_CUDA_TRY(cudaMallocHost(&p, bytes));
    return CMB_OK;
  }
};

// bytes of the cmb_fill_bytes stream of `seed`, generated on the host.
void host_seeded_bytes(uint8_t *dst, size_t bytes, uint64_t seed) {
  size_t i = 0;
  for (; i + 8 <= bytes; i += 8) {
    const uint64_t w = splitmix64_host(seed, i / 8);
    std::memcpy(dst + i, &w, 8);
  }
  for (; i < bytes; ++i) dst[i] = static_cast<uint8_t>(splitmix64_host(seed, i / 8) >> (8 * (i & 7)));
}

int section_pcie() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== PCIe (pinned host <-> device) ===\n");
  // 64 MiB pinned buffer, 10 copies per timing (src/pcie.cu:55-97).  The
  // host-to-device copies carry seeded bytes, checked on the device against
  // the same stream generated there; the device-to-host copies carry another
  // seed's bytes, checked on the host.
  const size_t bytes = 64ull << 20;
  constexpr uint64_t kUpSeed = 0x9C1E, kDownSeed = 0x9C1F;
  PinnedBuf host;
  TRY(host.alloc(bytes));
  DevBuf dev, ref, count;
  TRY(dev.alloc(bytes));
  TRY(ref.alloc(bytes));
  TRY(count.alloc(sizeof(unsigned long long)));
  host_seeded_bytes(static_cast<uint8_t *>(host.p), bytes, kUpSeed);
  double h2d = 0, d2h = 0;
  TRY(time_median(
      [&]() -> int {
        for (int r = 0; r < 10; ++r)
          CMB_CUDA_TRY(cudaMemcpyAsync(dev.p, host.p, bytes, cudaMemcpyHostToDevice, nullptr));
        return CMB_OK;
      },
      2, 1, &h2d));
  TRY(cmb_fill_bytes(ref.as<uint8_t>(), bytes, kUpSeed, nullptr));
  TRY(cmb_compare_bytes(dev.p, ref.p, bytes, count.as<unsigned long long>(), nullptr));
  unsigned long long up_bad = 0;
  CMB_CUDA_TRY(cudaMemcpy(&up_bad, count.p, sizeof(up_bad), cudaMemcpyDeviceToHost));
  TRY(cmb_fill_bytes(dev.as<uint8_t>(), bytes, kDownSeed, nullptr));
  TRY(time_median(
      [&]() -> int {
        for (int r = 0; r < 10; ++r)
          CMB_CUDA_TRY(cudaMemcpyAsync(host.p, dev.p, bytes, cudaMemcpyDeviceToHost, nullptr));
        return CMB_OK;
      },
      2, 1, &d2h));
  std::vector<uint8_t> want(bytes);
  host_seeded_bytes(want.data(), bytes, kDownSeed);
  const bool down_ok = std::memcmp(want.data(), host.p, bytes) == 0;
  const double up = gib_per_s(10.0 * bytes, h2d), down = gib_per_s(10.0 * bytes, d2h);
  printf("  HtoD pinned bandwidth: %.2f GiB/s (%s)\n  DtoH pinned bandwidth: %.2f GiB/s (%s)\n",
         up, up_bad == 0 ? "bytes verified" : "MISMATCH", down, down_ok ? "bytes verified" : "MISMATCH");
  if (up_bad != 0)
    return fail(CMB_ERR_MISMATCH, "PCIe: %llu words differ after the host-to-device copies", up_bad);
  if (!down_ok) return fail(CMB_ERR_MISMATCH, "PCIe: the device-to-host copies differ");
  g_results.log("pcie", "htod_bandwidth_GiB_s", up, "GiB/s");
  g_results.log("pcie", "dtoh_bandwidth_GiB_s", down, "GiB/s");
  g_results.log("pcie", "verified", 1.0, "bool");
  return CMB_OK;
}

int section_tma() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== TMA (cp.async.bulk.tensor) Probes ===\n");
  if (info.cc_major < 10) {
    // The B200 kernels are sm_100a code.
    g_results.log("tma", "tma_1d_load_latency_cyc", 0.0, "N/A");
    g_results.log("tma", "tma_g2s_load_bw_gibps", 0.0, "N/A");
    return fail(CMB_ERR_UNSUPPORTED, "TMA probes need an sm_100 device");
  }
  {
    // 1 KiB of hashed words; the reference's 16-byte load from coordinate
    // 0, 256 times, and the bytes it left in shared memory checked.
    DevBuf buf, cyc, st, landed;
    TRY(buf.alloc(1024));
    TRY(cyc.alloc(sizeof(uint32_t)));
    TRY(st.alloc(sizeof(int)));
    TRY(landed.alloc(16));
    TRY(cmb_fill_hash_u32(buf.as<uint32_t>(), 256, nullptr));
    const int iters = 256;
    TRY(cmb_tma_1d_latency(buf.p, 1024, 0, iters, cyc.as<uint32_t>(), landed.as<uint8_t>(),
                           st.as<int>(), nullptr));
    uint32_t h = 0;
    int status = 0;
    uint8_t got[16], want[16];
    CMB_CUDA_TRY(cudaMemcpy(&h, cyc.p, sizeof(h), cudaMemcpyDeviceToHost));
    CMB_CUDA_TRY(cudaMemcpy(&status, st.p, sizeof(status), cudaMemcpyDeviceToHost));
    CMB_CUDA_TRY(cudaMemcpy(got, landed.p, 16, cudaMemcpyDeviceToHost));
    CMB_CUDA_TRY(cudaMemcpy(want, buf.p, 16, cudaMemcpyDeviceToHost));
    if (status != 0) return fail(status, "TMA 1-D latency: a bounded wait expired");
    if (std::memcmp(got, want, 16) != 0)
      return fail(CMB_ERR_MISMATCH, "TMA 1-D latency: the landed bytes differ from the source");
    printf("  TMA 1D 16-byte load issue/wait cost: %.2f cycles (landed bytes verified)\n",
           (double)h / iters);
    g_results.log("tma", "tma_1d_load_latency_cyc", (double)h / iters, "cycles");
    g_results.log("tma", "tma_1d_verified", 1.0, "bool");
  }
  // 16384 x 16384 bf16, 128 x 128 boxes, 4-stage ring.
  const int n = 16384;
  const size_t bytes = (size_t)n * n * 2;
  DevBuf src, dst, xo, st;
  TRY(src.alloc(bytes));
  TRY(dst.alloc(bytes));
  TRY(xo.alloc(4096 * sizeof(uint32_t)));
  TRY(st.alloc(sizeof(int)));
  TRY(cmb_fill_normal_bf16(src.as<uint16_t>(), (size_t)n * n, kStreamSeed, 1.0f, nullptr));
  double lms = 0, cms = 0;
  TRY(time_median(
      [&] {
        return cmb_tma_tile_load_bf16(src.p, n, n, 128, 128, 4, xo.as<uint32_t>(), 4096,
                                      st.as<int>(), nullptr);
      },
      6, 1, &lms));
  TRY(time_median(
      [&] {
        return cmb_tma_tile_copy_bf16(dst.p, src.p, n, n, 128, 128, 4, 1, st.as<int>(), nullptr);
      },
      6, 1, &cms));
  int status = 0;
  CMB_CUDA_TRY(cudaMemcpy(&status, st.p, sizeof(status), cudaMemcpyDeviceToHost));
  if (status != 0) return fail(status, "TMA tile probe: a bounded wait expired");
  bool eq = false;
  TRY(expect_equal(src.p, dst.p, bytes, &eq));
  if (!eq) return fail(CMB_ERR_MISMATCH, "TMA tile copy output differs from its input");
  const double g2s = gib_per_s((double)bytes, lms);
  printf("  TMA G2S tile load BW: %.2f GiB/s; tile copy %.2f GB/s (read+write, bit-exact)\n", g2s,
         gb_per_s(2.0 * bytes, cms));
  g_results.log("tma", "tma_g2s_load_bw_gibps", g2s, "GiB/s");
  g_results.log("tma", "tile_copy_bw_gbps", gb_per_s(2.0 * bytes, cms), "GB/s");
  g_results.log("tma", "tile_copy_frac_of_8tbs_spec", gb_per_s(2.0 * bytes, cms) / 8000.0, "");
  g_results.log("tma", "tile_copy_verified", 1.0, "bool");
  g_results.log("tma", "tile_seed", static_cast<double>(kStreamSeed), "seed");
  g_results.log("tma", "tile_box_rows", 128, "");
  g_results.log("tma", "tile_box_cols", 128, "");
  g_results.log("tma", "tile_stages", 4, "");
  return CMB_OK;
}

namespace {

// Legacy mma.sync latency (one warp) and throughput, logged under `section`
// with the reference's key names.
int mma_sync_probe(const DeviceInfo &info, int kind, const char *section, const char *label,
                   double ops_per_mma, int k, bool int_ops, double *rate_out) {
  const int iters = 4096;
  DevBuf cyc, val;
  TRY(cyc.alloc(sizeof(uint64_t)));
  TRY(val.alloc(sizeof(double) * (size_t)info.sm_count * 4 * 8));
  TRY(cmb_mma_sync_latency(kind, iters, cyc.as<uint64_t>(), val.as<double>(), nullptr));
  uint64_t c = 0;
  CMB_CUDA_TRY(cudaMemcpy(&c, cyc.p, sizeof(c), cudaMemcpyDeviceToHost));
  const double lat = (double)c / iters;
  const int blocks = info.sm_count * 4, warps = 8;
  double ms = 0;
  TRY(time_median([&] { return cmb_mma_sync_throughput(kind, iters, blocks, warps, val.as<double>(), nullptr); },
                  3, 1, &ms));
  double v = 0;
  CMB_CUDA_TRY(cudaMemcpy(&v, val.p, sizeof(v), cudaMemcpyDeviceToHost));
  // four independent chains of `iters` MMAs, each adding k per MMA (the
  // f16 accumulator saturates, so it is not checked)
  const bool checked = kind != 1;
  if (checked && v != 4.0 * k * iters)
    return fail(CMB_ERR_MISMATCH, "%s: accumulator %.1f != %.1f", label, v, 4.0 * k * iters);
  const double ops = (double)blocks * warps * iters * 4 * ops_per_mma;
  const double rate = ops / (ms * 1e-3) / 1e12;
  printf("  %-18s latency %.2f cycles, throughput %.2f %s\n", label, lat, rate,
         int_ops ? "TOP/s" : "TFLOP/s");
  const std::string l(label), s(section);
  if (s == "tensor_core") {
    g_results.log(s, l + "_latency_cyc", lat, "cycles");
    g_results.log(s, l + "_latency_ns", nominal_ns(lat, info.clock_rate_khz), "nominal ns");
    g_results.log(s, l + "_throughput_tflops", rate, "TFLOP/s");
  } else {
    g_results.log(s, l + "_latency_cycles", lat, "cycles");
    g_results.log(s, l + "_latency_ns", nominal_ns(lat, info.clock_rate_khz), "ns");
    g_results.log(s, l + (int_ops ? "_throughput_Tops" : "_throughput_TFs"), rate,
                  int_ops ? "TOP/s" : "TFLOP/s");
  }
  if (rate_out != nullptr) *rate_out = rate;
  return CMB_OK;
}

}  // namespace

int section_tensor_core() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== Tensor Core Benchmarks ===\n");
  double tf32 = 0;
  TRY(mma_sync_probe(info, 0, "tensor_core", "mma_m16n8k8", 2.0 * 16 * 8 * 8, 8, false, &tf32));
  // the reference records its mma.sync TF32 rate as the TF32 peak
  // (src/tensor_core.cu:116-117)
  g_results.log("peak", "tf32_tensor_tflops", tf32, "TFLOP/s");
  // tcgen05 ceiling with resident shared-memory operands.
  DevBuf out, st;
  TRY(out.alloc((size_t)info.sm_count * 128 * sizeof(float)));
  TRY(st.alloc(sizeof(int)));
  for (int fp8 = 0; fp8 < 2; ++fp8) {
    const int iters = 8192;
    double ms = 0;
    TRY(time_median(
        [&] { return cmb_mma_rate(fp8, iters, info.sm_count, out.as<float>(), nullptr, st.as<int>(), nullptr); },
        4, 1, &ms));
    int status = 0;
    CMB_CUDA_TRY(cudaMemcpy(&status, st.p, sizeof(status), cudaMemcpyDeviceToHost));
    if (status != 0) return fail(status, "tcgen05 issue-rate probe failed its check");
    const double flop = (double)info.sm_count * iters * 4 * 2.0 * 128 * 256 * (fp8 ? 32 : 16);
    const double tf = flop / (ms * 1e-3) / 1e12;
    printf("  tcgen05 %s M=128 N=256 issue rate: %.1f TFLOP/s\n", fp8 ? "e4m3" : "bf16", tf);
    g_results.log("tensor_core_tcgen05", fp8 ? "fp8_issue_rate_tflops" : "bf16_issue_rate_tflops",
                  tf, "TFLOP/s");
  }
  return CMB_OK;
}

int section_tensor_core_extended() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  printf("=== Tensor Core Extended ===\n");
  double fp16_tf = 0;
  TRY(mma_sync_probe(info, 1, "tensor_core_extended", "fp16_m16n8k16", 2.0 * 16 * 8 * 16, 16, false, &fp16_tf));
  TRY(mma_sync_probe(info, 2, "tensor_core_extended", "bf16_m16n8k16", 2.0 * 16 * 8 * 16, 16, false, nullptr));
  TRY(mma_sync_probe(info, 3, "tensor_core_extended", "fp8_m16n8k32", 2.0 * 16 * 8 * 32, 32, false, nullptr));
  TRY(mma_sync_probe(info, 4, "tensor_core_extended", "int8_m16n8k32", 2.0 * 16 * 8 * 32, 32, true, nullptr));
  // the reference reports its FP16 mma.sync rate as the FP16 tensor peak
  // (src/tensor_core_extended.cu:289-290)
  g_results.log("peak", "fp16_tensor_tflops", fp16_tf, "TFLOP/s (FP16 accumulation)");

  // tcgen05 GEMM 8192^3, BF16 and FP8 e4m3 (per-tensor scale).
  const int M = 8192, N = 8192, K = 8192;
  const double flop = 2.0 * M * N * K;
  DevBuf A, B, C, qa, qb, sa, sb, st;
  TRY(A.alloc((size_t)M * K * 2));
  TRY(B.alloc((size_t)N * K * 2));
  TRY(C.alloc((size_t)M * N * 4));
  TRY(qa.alloc((size_t)M * K));
  TRY(qb.alloc((size_t)N * K));
  TRY(sa.alloc(2 * sizeof(float)));
  TRY(sb.alloc(2 * sizeof(float)));
  TRY(st.alloc(sizeof(int)));
  const float scale = 1.0f / std::sqrt((float)K);
  TRY(cmb_fill_normal_bf16(A.as<uint16_t>(), (size_t)M * K, kGemmSeed, scale, nullptr));
  TRY(cmb_fill_normal_bf16(B.as<uint16_t>(), (size_t)N * K, kGemmSeed + 1, scale, nullptr));
  TRY(cmb_quantize_e4m3(A.as<uint16_t>(), (size_t)M * K, qa.as<uint8_t>(), sa.as<float>(), nullptr));
  TRY(cmb_quantize_e4m3(B.as<uint16_t>(), (size_t)N * K, qb.as<uint8_t>(), sb.as<float>(), nullptr));
  std::vector<uint8_t> ha((size_t)M * K * 2), hb((size_t)N * K * 2);
  std::vector<float> hc((size_t)M * N);

  // Which die each SM sits on, measured; the GEMMs below run in the
  // die-split tile order with it (bit-identical to the plain order, which is
  // timed beside it).
  uint8_t die_map[CMB_DIE_MAP_IDS];
  int die_ids = 0;
  float near_far[2] = {0.f, 0.f};
  const int die_rc = cmb_sm_die_map(die_map, CMB_DIE_MAP_IDS, &die_ids, near_far, nullptr);
  if (die_rc == CMB_OK) {
    TRY(cmb_gemm_set_sm_die_map(die_map, die_ids));
    int on[2] = {0, 0};
    for (int i = 0; i < die_ids; ++i)
      if (die_map[i] <= 1) ++on[die_map[i]];
    printf("  SMs per die: %d + %d; cold load near / far die: %.0f / %.0f cycles\n", on[0], on[1],
           near_far[0], near_far[1]);
    g_results.log("tensor_core_tcgen05", "sms_on_die0", on[0], "count");
    g_results.log("tensor_core_tcgen05", "sms_on_die1", on[1], "count");
    g_results.log("tensor_core_tcgen05", "die_near_load_latency_cyc", near_far[0], "cycles");
    g_results.log("tensor_core_tcgen05", "die_far_load_latency_cyc", near_far[1], "cycles");
  } else {
    printf("  die map not measured (%s); GEMMs in the plain tile order\n", cmb_last_error());
    TRY(cmb_gemm_set_sm_die_map(nullptr, 0));
    for (const char *k : {"sms_on_die0", "sms_on_die1", "die_near_load_latency_cyc",
                          "die_far_load_latency_cyc"})
      g_results.log("tensor_core_tcgen05", k, 0.0, "N/A");
  }
  for (int fp8 = 0; fp8 < 2; ++fp8) {
    auto gemm = [&] {
      return fp8 ? cmb_gemm_e4m3(qa.p, qb.p, C.as<float>(), M, N, K, sa.as<float>(), sb.as<float>(), 2,
                                 st.as<int>(), nullptr)
                 : cmb_gemm_bf16(A.p, B.p, C.as<float>(), M, N, K, 2, st.as<int>(), nullptr);
    };
    double ms_plain = 0;
    if (die_rc == CMB_OK) {  // the plain order, for comparison
      TRY(cmb_gemm_set_sm_die_map(nullptr, 0));
      TRY(time_median(gemm, 6, 1, &ms_plain));
      TRY(cmb_gemm_set_sm_die_map(die_map, die_ids));
    }
    double ms = 0;
    TRY(time_median(gemm, 6, 1, &ms));
    int status = 0;
    CMB_CUDA_TRY(cudaMemcpy(&status, st.p, sizeof(status), cudaMemcpyDeviceToHost));
    if (status != 0) return fail(status, "tcgen05 GEMM: a bounded wait expired");
    const size_t eb = fp8 ? 1 : 2;
    CMB_CUDA_TRY(cudaMemcpy(ha.data(), fp8 ? qa.p : A.p, (size_t)M * K * eb, cudaMemcpyDeviceToHost));
    CMB_CUDA_TRY(cudaMemcpy(hb.data(), fp8 ? qb.p : B.p, (size_t)N * K * eb, cudaMemcpyDeviceToHost));
    CMB_CUDA_TRY(cudaMemcpy(hc.data(), C.p, hc.size() * 4, cudaMemcpyDeviceToHost));
    float hs[2] = {1.f, 1.f}, hs2[2] = {1.f, 1.f};
    if (fp8) {
      CMB_CUDA_TRY(cudaMemcpy(hs, sa.p, sizeof(hs), cudaMemcpyDeviceToHost));
      CMB_CUDA_TRY(cudaMemcpy(hs2, sb.p, sizeof(hs2), cudaMemcpyDeviceToHost));
    }
    // 64 sampled 256 x 256 output tiles against fp64 products
    const auto check0 = std::chrono::steady_clock::now();
    const double err = fp8 ? sampled_gemm_error<true>(ha, hb, hc, M, N, K, hs[0], hs2[0], 64)
                           : sampled_gemm_error<false>(ha, hb, hc, M, N, K, 1.0, 1.0, 64);
    if (!fp8) {  // the host reference's rate: fp64 products of those tiles, every host thread
      const double host_tf = 64.0 * 2.0 * 256 * 256 * K / seconds_since(check0) / 1e12;
      g_results.log("host_ref", "gemm_fp64_tiles_tflops", host_tf, "TFLOP/s");
    }
    const double tf = flop / (ms * 1e-3) / 1e12;
    const double spec = fp8 ? 4500.0 : 2250.0;
    const std::string p = fp8 ? "fp8_e4m3_gemm_8192" : "bf16_gemm_8192";
    printf("  tcgen05 %s GEMM 8192^3 (2-CTA 256x512): %.1f TFLOP/s (%.1f%% of %.0f), sampled "
           "rel err %.1e\n", fp8 ? "e4m3" : "bf16", tf, 100 * tf / spec, spec, err);
    if (err > 1e-2) return fail(CMB_ERR_MISMATCH, "%s: sampled rel err %.3g > 1e-2", p.c_str(), err);
    g_results.log("tensor_core_tcgen05", p + "_tflops", tf, "TFLOP/s");
    g_results.log("tensor_core_tcgen05", "gemm_seed", static_cast<double>(kGemmSeed), "seed");
    if (die_rc == CMB_OK) {
      const double tfp = flop / (ms_plain * 1e-3) / 1e12;
      printf("  (plain tile order: %.1f TFLOP/s)\n", tfp);
      g_results.log("tensor_core_tcgen05", p + "_plain_order_tflops", tfp, "TFLOP/s");
    } else {
      g_results.log("tensor_core_tcgen05", p + "_plain_order_tflops", 0.0, "N/A");
    }
    g_results.log("tensor_core_tcgen05", p + "_frac_of_spec", tf / spec, "");
    g_results.log("tensor_core_tcgen05", p + "_max_rel_err", err, "");
    g_results.log("tensor_core_tcgen05", p + "_verified", 1.0, "bool");

    // The same GEMM with bf16 C: timed, and checked to equal the fp32 C
    // above rounded to nearest-even bf16, element for element.
    DevBuf cb;
    TRY(cb.alloc((size_t)M * N * 2));
    double msb = 0;
    TRY(time_median(
        [&] {
          return cmb_gemm_bf16_out(fp8 ? qa.p : A.p, fp8 ? qb.p : B.p, cb.p, M, N, K, fp8,
                                   fp8 ? sa.as<float>() : nullptr, fp8 ? sb.as<float>() : nullptr,
                                   st.as<int>(), nullptr);
        },
        6, 1, &msb));
    CMB_CUDA_TRY(cudaMemcpy(&status, st.p, sizeof(status), cudaMemcpyDeviceToHost));
    if (status != 0) return fail(status, "tcgen05 GEMM (bf16 C): a bounded wait expired");
    std::vector<uint16_t> hcb((size_t)M * N);
    CMB_CUDA_TRY(cudaMemcpy(hcb.data(), cb.p, hcb.size() * 2, cudaMemcpyDeviceToHost));
    size_t bad = 0;
    for (size_t i = 0; i < hcb.size(); ++i) {
      uint32_t u;
      std::memcpy(&u, &hc[i], 4);
      const uint16_t rne = static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
      bad += hcb[i] != rne;
    }
    const double tfb = flop / (msb * 1e-3) / 1e12;
    printf("  tcgen05 %s GEMM 8192^3, bf16 C: %.1f TFLOP/s, %s\n", fp8 ? "e4m3" : "bf16", tfb,
           bad == 0 ? "equal to the fp32 C rounded to bf16" : "MISMATCH");
    if (bad != 0)
      return fail(CMB_ERR_MISMATCH, "%s: %zu bf16 outputs differ from the rounded fp32 C",
                  p.c_str(), bad);
    g_results.log("tensor_core_tcgen05", p + "_bf16out_tflops", tfb, "TFLOP/s");
    g_results.log("tensor_core_tcgen05", p + "_bf16out_verified", 1.0, "bool");
  }
  return CMB_OK;
}

namespace {

// Per-GPU state of the multi-GPU section: one host thread drives all GPUs,
// each launch is asynchronous, and every GPU's work is timed with its own
// events; a step's time is the slowest GPU's.
struct GpuSide {
  int dev = 0;
  void *send = nullptr, *recv = nullptr, *scratch = nullptr, *count = nullptr;
  int *count_status = nullptr;  // status word of the bulk-copy kernel
  cudaEvent_t a = nullptr, b = nullptr;
};

int free_sides(std::vector<GpuSide> &g) {
  for (auto &s : g) {
    cudaSetDevice(s.dev);
    for (void *p : {s.send, s.recv, s.scratch, s.count, static_cast<void *>(s.count_status)})
      if (p) cudaFree(p);
    if (s.a) cudaEventDestroy(s.a);
    if (s.b) cudaEventDestroy(s.b);
  }
  return CMB_OK;
}

// Launches one exchange step on every GPU; returns the max device time.
// How a P2P step moves bytes: in-kernel peer stores, in-kernel bulk copies,
// or the copy engines.
enum class P2PMethod { kStore, kBulk, kCopyEngine };

const char *p2p_method_name(P2PMethod m) {
  return m == P2PMethod::kStore ? "store" : m == P2PMethod::kBulk ? "bulk" : "copy_engine";
}

int p2p_step(std::vector<GpuSide> &g, size_t bytes, bool alltoall, P2PMethod method,
             double *ms_out) {
  const int n = static_cast<int>(g.size());
  for (auto &s : g) {
    CMB_CUDA_TRY(cudaSetDevice(s.dev));
    void *dst[8];
    const void *src[8];
    size_t nb[8];
    int jobs = 0;
    if (!alltoall) {
      dst[0] = g[(s.dev + 1) % n].recv;
      src[0] = s.send;
      nb[0] = bytes;
      jobs = 1;
    } else {
      // Staggered: GPU d visits peers d+1, d+2, ... and its own chunk last,
      // so at each position of the job list every GPU has one sender.
      const size_t c = bytes / n;
      for (int k = 0; k < n; ++k) {
        const int j = (s.dev + 1 + k) % n;
        dst[k] = static_cast<char *>(g[j].recv) + (size_t)s.dev * c;
        src[k] = static_cast<const char *>(s.send) + (size_t)j * c;
        nb[k] = c;
      }
      jobs = n;
    }
    CMB_CUDA_TRY(cudaEventRecord(s.a, nullptr));
    if (method == P2PMethod::kStore) TRY(cmb_p2p_scatter_store(dst, src, nb, jobs, 0, nullptr));
    else if (method == P2PMethod::kBulk)
      TRY(cmb_p2p_scatter_bulk(dst, src, nb, jobs, 0, s.count_status, nullptr));
    else TRY(cmb_p2p_scatter_copy_engine(dst, src, nb, jobs, nullptr));
    CMB_CUDA_TRY(cudaEventRecord(s.b, nullptr));
  }
  double worst = 0;
  for (auto &s : g) {
    CMB_CUDA_TRY(cudaSetDevice(s.dev));
    CMB_CUDA_TRY(cudaEventSynchronize(s.b));
    float t = 0;
    CMB_CUDA_TRY(cudaEventElapsedTime(&t, s.a, s.b));
    worst = std::max(worst, (double)t);
  }
  *ms_out = worst;
  return CMB_OK;
}

// Checks every GPU's receive buffer against the senders' seeded bytes.
int p2p_verify(std::vector<GpuSide> &g, size_t bytes, bool alltoall, uint64_t seed, bool *ok) {
  const int n = static_cast<int>(g.size());
  *ok = true;
  for (auto &s : g) {
    CMB_CUDA_TRY(cudaSetDevice(s.dev));
    for (int i = 0; i < (alltoall ? n : 1); ++i) {
      const int from = alltoall ? i : (s.dev - 1 + n) % n;
      const size_t c = alltoall ? bytes / n : bytes;
      const size_t recv_off = alltoall ? (size_t)i * c : 0, src_off = alltoall ? (size_t)s.dev * c : 0;
      TRY(cmb_fill_bytes(static_cast<uint8_t *>(s.scratch), bytes, seed + from, nullptr));
      TRY(cmb_compare_bytes(static_cast<char *>(s.recv) + recv_off,
                            static_cast<char *>(s.scratch) + src_off, c,
                            static_cast<unsigned long long *>(s.count), nullptr));
      unsigned long long h = 1;
      CMB_CUDA_TRY(cudaMemcpy(&h, s.count, sizeof(h), cudaMemcpyDeviceToHost));
      *ok = *ok && (h == 0);
    }
  }
  return CMB_OK;
}

int multi_gpu_body(std::vector<GpuSide> &g, size_t bytes) {
  const uint64_t seed = kStreamSeed;
  const int n = static_cast<int>(g.size());
  for (auto &s : g) {
    CMB_CUDA_TRY(cudaSetDevice(s.dev));
    for (auto &o : g)
      if (o.dev != s.dev) TRY(cmb_p2p_enable_peer(o.dev));
    CMB_CUDA_TRY(cudaMalloc(&s.send, bytes));
    CMB_CUDA_TRY(cudaMalloc(&s.recv, bytes));
    CMB_CUDA_TRY(cudaMalloc(&s.scratch, bytes));
    CMB_CUDA_TRY(cudaMalloc(&s.count, sizeof(unsigned long long)));
    CMB_CUDA_TRY(cudaMalloc(&s.count_status, sizeof(int)));
    CMB_CUDA_TRY(cudaEventCreate(&s.a));
    CMB_CUDA_TRY(cudaEventCreate(&s.b));
    TRY(cmb_fill_bytes(static_cast<uint8_t *>(s.send), bytes, seed + s.dev, nullptr));
  }
  for (auto &s : g) {
    CMB_CUDA_TRY(cudaSetDevice(s.dev));
    CMB_CUDA_TRY(cudaDeviceSynchronize());
  }
  for (int alltoall = 0; alltoall < 2; ++alltoall) {
    for (P2PMethod method : {P2PMethod::kStore, P2PMethod::kBulk, P2PMethod::kCopyEngine}) {
      std::vector<double> ms;
      for (auto &s : g) {
        CMB_CUDA_TRY(cudaSetDevice(s.dev));
        CMB_CUDA_TRY(cudaMemset(s.count_status, 0, sizeof(int)));
      }
      for (int r = 0; r < 6; ++r) {
        double t = 0;
        TRY(p2p_step(g, bytes, alltoall != 0, method, &t));
        if (r > 0) ms.push_back(t);
      }
      for (auto &s : g) {
        CMB_CUDA_TRY(cudaSetDevice(s.dev));
        int st = 0;
        CMB_CUDA_TRY(cudaMemcpy(&st, s.count_status, sizeof(int), cudaMemcpyDeviceToHost));
        if (st != 0)
          return fail(st, "p2p %s on device %d: kernel status %d (%s)", p2p_method_name(method),
                      s.dev, st, cmb_status_string(st));
      }
      std::sort(ms.begin(), ms.end());
      const double t = ms[ms.size() / 2];
      bool ok = false;
      TRY(p2p_verify(g, bytes, alltoall != 0, seed, &ok));
      if (!ok) return fail(CMB_ERR_MISMATCH, "p2p %s: received bytes differ", alltoall ? "all-to-all" : "ring");
      const double egress = alltoall ? (double)bytes * (n - 1) / n : (double)bytes;
      const double link = gb_per_s(egress, t);
      const std::string k = std::string(alltoall ? "alltoall_" : "ring_") + p2p_method_name(method);
      printf("  %-22s %d GPUs: %.1f GB/s egress per GPU (%.1f%% of 900), %.1f GB/s aggregate, bit-exact\n",
             k.c_str(), n, link, 100 * link / 900.0, n * link);
      g_results.log("p2p", k + "_link_gbps", link, "GB/s");
      g_results.log("p2p", k + "_aggregate_gbps", n * link, "GB/s");
      g_results.log("p2p", k + "_frac_of_900", link / 900.0, "");
      g_results.log("p2p", k + "_verified", 1.0, "bool");
    }
  }
  // Sharded copy stream: every GPU copies its own buffer at once.
  std::vector<double> ms;
  for (int r = 0; r < 6; ++r) {
    for (auto &s : g) {
      CMB_CUDA_TRY(cudaSetDevice(s.dev));
      CMB_CUDA_TRY(cudaEventRecord(s.a, nullptr));
      TRY(cmb_stream_copy(s.scratch, s.send, bytes, nullptr));
      CMB_CUDA_TRY(cudaEventRecord(s.b, nullptr));
    }
    double worst = 0;
    for (auto &s : g) {
      CMB_CUDA_TRY(cudaSetDevice(s.dev));
      CMB_CUDA_TRY(cudaEventSynchronize(s.b));
      float t = 0;
      CMB_CUDA_TRY(cudaEventElapsedTime(&t, s.a, s.b));
      worst = std::max(worst, (double)t);
    }
    if (r > 0) ms.push_back(worst);
  }
  std::sort(ms.begin(), ms.end());
  const double agg = gb_per_s(2.0 * bytes * n, ms[ms.size() / 2]);
  printf("  sharded copy stream, %d GPUs: %.1f GB/s aggregate\n", n, agg);
  g_results.log("p2p", "sharded_stream_aggregate_gbps", agg, "GB/s");
  g_results.log("p2p", "gpus_used", n, "");
  g_results.log("p2p", "seed", static_cast<double>(kStreamSeed), "seed");
  return CMB_OK;
}

}  // namespace

int section_multi_gpu() {
  DeviceInfo info;
  TRY(query_device(0, &info));
  int count = 0;
  CMB_CUDA_TRY(cudaGetDeviceCount(&count));
  printf("=== Multi-GPU (NVLink P2P) ===\n");
  int can = 0;
  if (count >= 2) CMB_CUDA_TRY(cudaDeviceCanAccessPeer(&can, 0, 1));
  // the reference's availability keys (src/pcie.cu:100-112)
  g_results.log("pcie", "device_count", count, "");
  g_results.log("pcie", "p2p_available", can ? 1.0 : 0.0, "bool");
  g_results.log("p2p", "device_count", count, "");
  if (count < 2 || !can) {
    printf("  %d device(s), peer access %s: nothing to exchange\n", count, can ? "yes" : "no");
    return CMB_OK;
  }
  std::vector<GpuSide> g(std::min(count, 8));
  for (int d = 0; d < (int)g.size(); ++d) g[d].dev = d;
  const int rc = multi_gpu_body(g, 256ull << 20);
  free_sides(g);
  cudaSetDevice(0);
  return rc;
}

namespace {
// The (section, key) paths the reference's results/report.html reads.
const char *const kReportKeys[][2] = {
#include "report_keys.inc"
};
}  // namespace

void log_report_placeholders() {
  for (const auto &k : kReportKeys)
    if (!g_results.has(k[0], k[1])) g_results.log(k[0], k[1], 0.0, "N/A");
}

size_t report_key_count() { return sizeof(kReportKeys) / sizeof(kReportKeys[0]); }

bool report_key(size_t i, const char **section, const char **key) {
  if (i >= report_key_count()) return false;
  *section = kReportKeys[i][0];
  *key = kReportKeys[i][1];
  return true;
}

namespace {

struct Section {
  const char *flag, *help;
  int (*run)();
};

const Section kSections[] = {
    {"--device", "Device / SM info and derived peaks", section_device_info},
    {"--memory", "HBM read/copy streams and DRAM pointer chase", section_global_memory},
    {"--cache", "L1/L2 dependent-load latency sweep", section_cache},
    {"--memory-more", "L2 aggregate read bandwidth", section_memory_more},
    {"--pcie", "Pinned host <-> device copy bandwidth", section_pcie},
    {"--tma", "TMA bulk-tensor latency, tile load and tile copy", section_tma},
    {"--tensor", "mma.sync TF32 and tcgen05 issue-rate probes", section_tensor_core},
    {"--tensor-ext", "mma.sync FP16/BF16/FP8/INT8 and tcgen05 BF16/FP8 GEMM", section_tensor_core_extended},
    {"--p2p", "Multi-GPU sharded stream and NVLink peer copies", section_multi_gpu},
};

void usage(const char *name) {
  printf("Usage: %s [option]...\nOptions:\n", name);
  for (const auto &s : kSections) printf("  %-14s %s\n", s.flag, s.help);
  printf("  %-14s %s\n", "--json", "Run all sections and write the results file");
  printf("  %-14s %s\n", "--all", "Run all sections (default)");
}

// Runs one section inside an NVTX range named by its flag, so a profiler's
// timeline (or ncu --nvtx-include) can pick a section out of a full run.
int run_section(const Section &s) {
  nvtxRangePushA(s.flag + 2);  // "--memory" -> "memory"
  const int rc = s.run();
  nvtxRangePop();
  return rc;
}

int run_all() {
  for (const auto &s : kSections) {
    const int rc = run_section(s);
    if (rc != CMB_OK) return rc;
  }
  log_report_placeholders();
  return CMB_OK;
}

int report_failure(int rc) {
  fprintf(stderr, "cmb_b200: %s: %s\n", cmb_status_string(rc), cmb_last_error());
  return 1;
}

int write_results(const char *path) {
  std::string err;
  if (!g_results.writeJson(path, &err)) {
    fprintf(stderr, "%s\n", err.c_str());
    return 1;
  }
  return 0;
}

}  // namespace

int run_cli(int argc, const char *const *argv, const char *json_path) {
  if (argc <= 1) {
    const int rc = run_all();
    if (rc != CMB_OK) return report_failure(rc);
    return write_results(json_path);
  }
  bool ok = true, ran = false;
  for (int i = 1; i < argc; ++i) {
    const char *opt = argv[i];
    if (std::strcmp(opt, "--help") == 0 || std::strcmp(opt, "-h") == 0) {
      usage("cmb_b200");
      ran = true;
      continue;
    }
    int rc = -1;
    if (std::strcmp(opt, "--all") == 0 || std::strcmp(opt, "--json") == 0) {
      rc = run_all();
    } else {
      for (const auto &s : kSections)
        if (std::strcmp(opt, s.flag) == 0) rc = run_section(s);
    }
    if (rc == -1) {
      printf("Unknown option: %s\n", opt);
      usage(argv[0]);
      ok = false;
    } else if (rc != CMB_OK) {
      return report_failure(rc);
    } else {
      ran = true;
    }
  }
  if (ran && ok && g_results.hasDevice()) {
    if (write_results(json_path) != 0) return 1;
  }
  return ok ? 0 : 1;
}

}  // namespace cmb

using namespace cmb;

extern "C" int cmb_benchmark_global_memory(void) { return section_global_memory(); }
extern "C" int cmb_benchmark_cache(void) { return section_cache(); }
extern "C" int cmb_benchmark_tma(void) { return section_tma(); }
extern "C" int cmb_benchmark_tensor_core(void) { return section_tensor_core(); }
extern "C" int cmb_benchmark_tensor_core_extended(void) { return section_tensor_core_extended(); }
extern "C" int cmb_benchmark_multi_gpu(void) { return section_multi_gpu(); }
extern "C" int cmb_benchmark_memory_more(void) { return section_memory_more(); }
extern "C" int cmb_benchmark_pcie(void) { return section_pcie(); }
extern "C" int cmb_results_log_report_placeholders(void) {
  log_report_placeholders();
  return CMB_OK;
}
extern "C" size_t cmb_report_key_count(void) { return report_key_count(); }
extern "C" int cmb_report_key(size_t i, const char **section, const char **key) {
  if (section == nullptr || key == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_report_key: null output pointer");
  if (!report_key(i, section, key))
    return fail(CMB_ERR_INVALID_ARG, "cmb_report_key: index %zu >= %zu keys", i,
                report_key_count());
  return CMB_OK;
}
extern "C" int cmb_run_cli(int argc, const char *const *argv, const char *json_path) {
  return run_cli(argc, argv, json_path ? json_path : "results/results.json");
}
