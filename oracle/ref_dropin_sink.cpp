// ref_dropin_sink.cpp — test infrastructure: the one file a reference build
// adds when it links libcmb_b200.so in place of its own probe sections.
// It installs a results sink so the library's sections log into the
// reference's cmb::g_results (include/result_logger.h:111-144), which the
// reference's main.cu writes to results/results.json with its own writer
// (src/result_logger.cu:10-43).  Compiled against the reference's headers by
// oracle/Makefile target `ref-dropin`; nothing in the library depends on it.
#include "cmb_b200.h"
#include "result_logger.h"

namespace {

void forward_log(const char *section, const char *key, double value, const char *unit, void *) {
  cmb::g_results.log(section, key, value, unit);
}

void forward_device(const char *name, const char *arch, int sm_count, int clock_khz,
                    int mem_clock_khz, int mem_bus_width, void *) {
  cmb::g_results.setDevice(name, arch, sm_count, clock_khz, mem_clock_khz, mem_bus_width);
}

// Runs during the executable's static initialisation, after the library's
// (a shared library is initialised before the program that needs it).
const int g_sink_installed = cmb_results_set_sink(forward_log, forward_device, nullptr);

}  // namespace
