// main.cpp — the cmb_b200 CLI: the reference's section flags
// (src/main.cu:65-152), results written to results/results.json relative to
// the working directory (src/main.cu:61-63), or to --out=<path>.
#include <sys/stat.h>

#include <cstring>
#include <string>
#include <vector>

#include "sections.h"

int main(int argc, char **argv) {
  std::string out = "results/results.json";
  std::vector<const char *> args = {argv[0]};
  for (int i = 1; i < argc; ++i) {
    if (std::strncmp(argv[i], "--out=", 6) == 0) out = argv[i] + 6;
    else args.push_back(argv[i]);
  }
  const size_t slash = out.rfind('/');
  if (slash != std::string::npos && slash > 0) mkdir(out.substr(0, slash).c_str(), 0755);
  return cmb::run_cli(static_cast<int>(args.size()), args.data(), out.c_str());
}
