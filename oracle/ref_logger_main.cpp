// Driver around the reference's own ResultLogger (src/result_logger.cu,
// include/result_logger.h), compiled from the reference sources in place by
// oracle/Makefile (target `ref`).  Test infrastructure: it turns a script of
// logger calls on stdin into the JSON the reference would write, so the
// committed golden files pin this repository's logger byte for byte.
//
// Script lines (tab separated):
//   D <name> <arch> <sm_count> <clock_khz> <mem_clock_khz> <bus_bits>
//   L <section> <key> <value> <unit>      (unit may be empty)
//   W <path>
#include "result_logger.h"

#include <cstdlib>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

static std::vector<std::string> split_tabs(const std::string &line) {
  std::vector<std::string> out;
  std::string cur;
  for (char c : line) {
    if (c == '\t') { out.push_back(cur); cur.clear(); }
    else cur += c;
  }
  out.push_back(cur);
  return out;
}

int main() {
  std::string line;
  while (std::getline(std::cin, line)) {
    if (line.empty()) continue;
    std::vector<std::string> f = split_tabs(line);
    if (f[0] == "D" && f.size() == 7) {
      cmb::g_results.setDevice(f[1], f[2], std::atoi(f[3].c_str()), std::atoi(f[4].c_str()),
                               std::atoi(f[5].c_str()), std::atoi(f[6].c_str()));
    } else if (f[0] == "L" && f.size() >= 4) {
      cmb::g_results.log(f[1], f[2], std::strtod(f[3].c_str(), nullptr), f.size() > 4 ? f[4] : "");
    } else if (f[0] == "W" && f.size() == 2) {
      cmb::g_results.writeJson(f[1]);
    } else {
      std::cerr << "bad script line: " << line << "\n";
      return 2;
    }
  }
  return 0;
}
