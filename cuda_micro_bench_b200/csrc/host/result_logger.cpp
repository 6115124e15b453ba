// result_logger.cpp — results table and its JSON serialisation.
#include "result_logger.h"

#include <cerrno>
#include <cstdio>
#include <cstring>

#include "../../../include/cmb_b200.h"
#include "../cmb_host.h"

namespace cmb {

ResultLogger g_results;

void ResultLogger::setDevice(const std::string &name, const std::string &arch, int sm_count,
                             int clock_khz, int mem_clock_khz, int mem_bus_width) {
  std::lock_guard<std::mutex> lock(mu_);
  device_ = name;
  arch_ = arch;
  sm_count_ = sm_count;
  clock_khz_ = clock_khz;
  mem_clock_khz_ = mem_clock_khz;
  mem_bus_width_ = mem_bus_width;
  if (sink_device_ != nullptr)
    sink_device_(name.c_str(), arch.c_str(), sm_count, clock_khz, mem_clock_khz, mem_bus_width,
                 sink_user_);
}

void ResultLogger::log(const std::string &section, const std::string &key, double value,
                       const std::string &unit) {
  std::lock_guard<std::mutex> lock(mu_);
  sections_[section][key] = Entry{value, unit};
  if (sink_log_ != nullptr) sink_log_(section.c_str(), key.c_str(), value, unit.c_str(), sink_user_);
}

void ResultLogger::setSink(cmb_results_log_fn log, cmb_results_device_fn device, void *user) {
  std::lock_guard<std::mutex> lock(mu_);
  sink_log_ = log;
  sink_device_ = device;
  sink_user_ = user;
}

bool ResultLogger::hasDevice() const {
  std::lock_guard<std::mutex> lock(mu_);
  return !device_.empty();
}

bool ResultLogger::has(const std::string &section, const std::string &key) const {
  std::lock_guard<std::mutex> lock(mu_);
  auto it = sections_.find(section);
  return it != sections_.end() && it->second.count(key) != 0;
}

void ResultLogger::clear() {
  std::lock_guard<std::mutex> lock(mu_);
  device_.clear();
  arch_.clear();
  sm_count_ = clock_khz_ = mem_clock_khz_ = mem_bus_width_ = 0;
  sections_.clear();
}

namespace {

// String values escape quote, backslash, newline, CR and tab; keys are
// written as given (the reference writes keys unescaped).
std::string quoted(const std::string &s) {
  std::string r = "\"";
  for (char c : s) {
    switch (c) {
      case '"': r += "\\\""; break;
      case '\\': r += "\\\\"; break;
      case '\n': r += "\\n"; break;
      case '\r': r += "\\r"; break;
      case '\t': r += "\\t"; break;
      default: r += c;
    }
  }
  return r + "\"";
}

std::string pad(int n) { return std::string(static_cast<size_t>(n), ' '); }

}  // namespace

std::string ResultLogger::toJson() const {
  std::lock_guard<std::mutex> lock(mu_);
  std::string o = "{\n";
  o += pad(2) + "\"device\": " + quoted(device_) + ",\n";
  o += pad(2) + "\"architecture\": " + quoted(arch_) + ",\n";
  o += pad(2) + "\"sm_count\": " + std::to_string(sm_count_) + ",\n";
  o += pad(2) + "\"clock_khz\": " + std::to_string(clock_khz_) + ",\n";
  o += pad(2) + "\"memory_clock_khz\": " + std::to_string(mem_clock_khz_) + ",\n";
  o += pad(2) + "\"memory_bus_width_bits\": " + std::to_string(mem_bus_width_) + ",\n";
  o += pad(2) + "\"results\": {\n";
  size_t si = 0;
  for (const auto &sec : sections_) {
    o += pad(4) + "\"" + sec.first + "\": {\n";
    size_t ki = 0;
    for (const auto &kv : sec.second) {
      o += pad(6) + "\"" + kv.first + "\": {\n";
      o += pad(8) + "\"value\": " +
           (kv.second.unit == "N/A" ? std::string("null") : std::to_string(kv.second.value)) +
           ",\n";
      o += pad(8) + "\"unit\": " + quoted(kv.second.unit) + "\n";
      o += pad(6) + "}" + (++ki < sec.second.size() ? ",\n" : "\n");
    }
    o += pad(4) + "}" + (++si < sections_.size() ? ",\n" : "\n");
  }
  o += pad(2) + "}\n";
  o += "}\n";
  return o;
}

bool ResultLogger::writeJson(const std::string &path, std::string *err) const {
  const std::string text = toJson();
  FILE *f = std::fopen(path.c_str(), "wb");
  if (f == nullptr) {
    if (err) *err = "Cannot open results path: " + path + " (" + std::strerror(errno) + ")";
    return false;
  }
  const size_t wrote = std::fwrite(text.data(), 1, text.size(), f);
  const bool ok = (wrote == text.size()) && (std::fclose(f) == 0);
  if (!ok && err) *err = "Cannot write results path: " + path;
  return ok;
}

}  // namespace cmb

using namespace cmb;

extern "C" int cmb_results_set_device(const char *name, const char *arch, int sm_count,
                                      int clock_khz, int mem_clock_khz, int mem_bus_width) {
  if (name == nullptr || arch == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_results_set_device: null name or arch");
  g_results.setDevice(name, arch, sm_count, clock_khz, mem_clock_khz, mem_bus_width);
  return CMB_OK;
}

extern "C" int cmb_results_log(const char *section, const char *key, double value,
                               const char *unit) {
  if (section == nullptr || key == nullptr)
    return fail(CMB_ERR_INVALID_ARG, "cmb_results_log: null section or key");
  g_results.log(section, key, value, unit ? unit : "");
  return CMB_OK;
}

extern "C" int cmb_results_write_json(const char *path) {
  if (path == nullptr) return fail(CMB_ERR_INVALID_ARG, "cmb_results_write_json: null path");
  std::string err;
  if (!g_results.writeJson(path, &err)) return fail(CMB_ERR_IO, "%s", err.c_str());
  return CMB_OK;
}

extern "C" int cmb_results_clear(void) {
  g_results.clear();
  return CMB_OK;
}

extern "C" int cmb_results_set_sink(cmb_results_log_fn log, cmb_results_device_fn device,
                                    void *user) {
  cmb::g_results.setSink(log, device, user);
  return CMB_OK;
}
