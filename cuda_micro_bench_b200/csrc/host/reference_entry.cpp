// reference_entry.cpp — the section entry points with the reference's own
// signatures and error behaviour, for linking into the reference's main.cu
// (src/main.cu:9-32 declares them, run_all and dispatch call them,
// src/main.cu:34-59,96-152).
//
// `void cmb::benchmark_<section>()` runs the section, logs its keys (into
// the library's table, and through the results sink of
// cmb_results_set_sink() into the host's table), and returns.  Like the
// reference, a failed CUDA call or self-check prints the reason and ends the
// process with EXIT_FAILURE (CUDA_CHECK, include/utils.h:11-19; the chase
// self-check, include/memory_chase.h:161-164), and a device without the
// needed feature logs its keys as "N/A" and returns (src/tma.cu:164-169).
//
// These six are the library's only exported C++ symbols: every other C++
// name stays inside the library (see exports.map), so a reference build's
// own cmb::g_results and cmb::ResultLogger never meet the library's.
#include <cstdio>
#include <cstdlib>

#include "../../../include/cmb_b200.h"
#include "sections.h"

namespace cmb {
namespace {

void run_or_exit(int (*section)(), const char *name) {
  const int rc = section();
  if (rc == CMB_OK) return;
  if (rc == CMB_ERR_UNSUPPORTED) {
    printf("  %s: skipped: %s\n", name, cmb_last_error());
    return;
  }
  fprintf(stderr, "%s failed: %s: %s\n", name, cmb_status_string(rc), cmb_last_error());
  exit(EXIT_FAILURE);
}

}  // namespace

void benchmark_global_memory() { run_or_exit(section_global_memory, "benchmark_global_memory"); }
void benchmark_cache() { run_or_exit(section_cache, "benchmark_cache"); }
void benchmark_tma() { run_or_exit(section_tma, "benchmark_tma"); }
void benchmark_tensor_core() { run_or_exit(section_tensor_core, "benchmark_tensor_core"); }
void benchmark_tensor_core_extended() {
  run_or_exit(section_tensor_core_extended, "benchmark_tensor_core_extended");
}
void benchmark_multi_gpu() { run_or_exit(section_multi_gpu, "benchmark_multi_gpu"); }

}  // namespace cmb
