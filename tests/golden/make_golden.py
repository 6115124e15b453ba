"""Generates the golden fixtures in this directory from the reference itself.

logger_*.script / logger_*.json
    Logger call scripts and the JSON that the reference's own ResultLogger
    (src/result_logger.cu, include/result_logger.h), compiled from the
    reference sources by `make -C oracle ref`, writes for them.  These pin
    cmb_results_* (the results.json writer) byte for byte.

report_keys.txt
    Every results key path the reference's HTML report reads
    (results/report.html, the ['results', section, key] lists of its
    tables), one "section key" per line: the CLI's full run must produce
    each of them.

Run here, where the reference tree is present:
    python tests/golden/make_golden.py
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

SCRIPTS = {
    # The keys benchmark_global_memory logs (src/mem_global.cu:59-74).
    "memory": [
        ("D", "NVIDIA B200", "10.0", "148", "1965000", "3996000", "8192"),
        ("L", "memory_dram", "read_bw_gibps", "5712.345678901", "GiB/s"),
        ("L", "memory_dram", "copy_max_bw_gibps", "5923.5", "GiB/s"),
        ("L", "memory", "dram_read_bw_gbps", "6133.74", "GB/s"),
        ("L", "memory_dram", "stream_working_set_bytes", "1073741824", "bytes"),
        ("L", "memory", "dram_latency_cyc", "1234.0000004", "cycles"),
        ("L", "memory_dram", "pointer_chase_latency_ns", "628.0", "nominal ns"),
        ("L", "memory_dram", "chase_working_set_bytes", "536870912", "bytes"),
        ("L", "memory_dram", "chase_loads_per_sample", "4194304", "loads"),
        ("L", "memory_dram", "chase_min_sector_footprint_bytes", "134217728", "bytes"),
    ],
    # N/A -> null, empty unit, negative and tiny values, last write wins,
    # escapes in string values, unescaped keys.
    "edge": [
        ("D", 'GPU "quoted"\\name', "10.0", "148", "0", "0", "0"),
        ("L", "tma", "tma_1d_load_latency_cyc", "0", "N/A"),
        ("L", "tma", "tma_g2s_load_bw_gibps", "-1.5e-7", ""),
        ("L", "peak", "fp32_tflops", "1e15", "TFLOP/s"),
        ("L", "peak", "fp32_tflops", "77.25", "TFLOP/s"),
        ("L", "a_section", "k", "3.0000005", "u\"q\"\\b"),
        ("L", "Z", "upper", "2", "x"),
    ],
    # No results at all.
    "empty": [
        ("D", "NVIDIA B200", "10.0", "148", "1965000", "3996000", "8192"),
    ],
}


# The reference checkout's report: CMB_REFERENCE_ROOT, or the `reference`
# directory beside this repository.
REPORT = os.path.join(
    os.environ.get("CMB_REFERENCE_ROOT")
    or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__))))), "reference"),
    "results", "report.html")


def report_keys():
    import re

    html = open(REPORT).read()
    pattern = re.compile(r"\[((?:\s*'[^']+'\s*,)*\s*'[^']+'\s*)\]", re.MULTILINE)
    keys = set()
    for m in pattern.findall(html):
        parts = [p.strip().strip("'") for p in m.split(",") if p.strip()]
        if len(parts) == 3 and parts[0] == "results":
            keys.add((parts[1], parts[2]))
    return sorted(keys)


def main() -> None:
    import oracle

    with open(os.path.join(HERE, "report_keys.txt"), "w") as f:
        for sec, key in report_keys():
            f.write(f"{sec} {key}\n")

    oracle.build(ref=True)
    for name, lines in SCRIPTS.items():
        script = os.path.join(HERE, f"logger_{name}.script")
        out = os.path.join(HERE, f"logger_{name}.json")
        text = "".join("\t".join(fields) + "\n" for fields in lines)
        with open(script, "w") as f:
            f.write(text)
        tmp = out + ".tmp"
        proc = subprocess.run([oracle.REF_LOGGER], input=text + f"W\t{tmp}\n", text=True)
        if proc.returncode != 0:
            raise SystemExit(f"reference logger failed on {name}")
        os.replace(tmp, out)
        print("wrote", out)


if __name__ == "__main__":
    main()
