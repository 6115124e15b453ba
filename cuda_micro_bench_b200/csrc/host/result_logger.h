// result_logger.h — the probe results table and its results.json writer.
//
// Same data model and file format as the reference's ResultLogger
// (include/result_logger.h:111-144, src/result_logger.cu:10-43): a device
// header plus section -> key -> {value, unit}, sections and keys in sorted
// order, the last write of a key wins, numbers printed like std::to_string
// (six decimals) and unit "N/A" written as a null value.  Unlike the
// reference it is safe to call from several host threads, and it can pass
// every entry on to a host's own table (the reference's g_results, when the
// library is linked into the reference's main.cu).
#pragma once

#include <map>
#include <mutex>
#include <string>

#include "../../../include/cmb_b200.h"

namespace cmb {

class ResultLogger {
 public:
  void setDevice(const std::string &name, const std::string &arch, int sm_count, int clock_khz,
                 int mem_clock_khz, int mem_bus_width);
  void log(const std::string &section, const std::string &key, double value,
           const std::string &unit = "");
  bool hasDevice() const;
  bool has(const std::string &section, const std::string &key) const;
  // Serialised table (the exact bytes writeJson stores).
  std::string toJson() const;
  // Returns false (and leaves the reason in `err`) if the file cannot be
  // written.
  bool writeJson(const std::string &path, std::string *err) const;
  void clear();
  // Every later setDevice/log is also passed to these callbacks (either may
  // be null), under the table's lock, so a host's own non-thread-safe
  // table sees one call at a time.
  void setSink(cmb_results_log_fn log, cmb_results_device_fn device, void *user);

 private:
  struct Entry {
    double value;
    std::string unit;
  };
  mutable std::mutex mu_;
  std::string device_, arch_;
  int sm_count_ = 0, clock_khz_ = 0, mem_clock_khz_ = 0, mem_bus_width_ = 0;
  std::map<std::string, std::map<std::string, Entry>> sections_;
  cmb_results_log_fn sink_log_ = nullptr;
  cmb_results_device_fn sink_device_ = nullptr;
  void *sink_user_ = nullptr;
};

// The process-wide table the probe sections log into.
extern ResultLogger g_results;

}  // namespace cmb
