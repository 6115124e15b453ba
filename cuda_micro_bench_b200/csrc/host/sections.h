// sections.h — the reference's probe sections on top of the C ABI.
//
// Same result keys as the reference's `void cmb::benchmark_<section>()`
// (src/main.cu:9-32): each section queries device 0, allocates its buffers,
// runs the B200 kernels through include/cmb_b200.h, checks their outputs,
// times them with CUDA events and logs into g_results.  The section_*
// functions return a cmb_status where the reference exits on a CUDA error
// (include/utils.h:11-19) or a failed self-check
// (include/memory_chase.h:161-164); the CLI turns a failure into exit code 1.
// reference_entry.cpp wraps them in the reference's own signatures and
// error behaviour (void, exit on failure) for the reference's main.cu.
#pragma once

#include <string>

namespace cmb {

struct DeviceInfo {
  int id = 0;
  std::string name;
  int cc_major = 0, cc_minor = 0;
  int sm_count = 0;
  int max_threads_per_sm = 0;
  int max_warps_per_sm = 0;
  int clock_rate_khz = 0;
  int memory_clock_khz = 0;
  int mem_bus_width = 0;
  int l2_cache_size = 0;
  size_t total_global_mem = 0;
  size_t shared_mem_per_block_optin = 0;
};

// Fills `info` for device `dev`, makes it current and records it as the
// results file's device header (include/utils.h:47-82).
int query_device(int dev, DeviceInfo *info);

int section_device_info();         // --device      (src/device_info.cu, header keys only)
int section_global_memory();       // --memory      (src/mem_global.cu:27-75)
int section_cache();               // --cache       (src/mem_cache.cu:4-24)
int section_memory_more();         // --memory-more (src/memory_more.cu:201-234, L2 only)
int section_pcie();                // --pcie        (src/pcie.cu:55-97, bandwidth only)
int section_tma();                 // --tma         (src/tma.cu:157-259)
int section_tensor_core();         // --tensor      (src/tensor_core.cu:66-120)
int section_tensor_core_extended();  // --tensor-ext (src/tensor_core_extended.cu:321-357)
int section_multi_gpu();           // --p2p         (new: sharded stream + NVLink P2P)

// Logs every results key the reference's report reads and no section
// measured, as "N/A" (null), so the report renders.
void log_report_placeholders();
// The report's key table: its size, and entry i (false past the end).
size_t report_key_count();
bool report_key(size_t i, const char **section, const char **key);

// The CLI (src/main.cu:156-181): flags run sections; no flags runs all and
// writes `json_path`.  Returns the process exit code.
int run_cli(int argc, const char *const *argv, const char *json_path);

}  // namespace cmb
