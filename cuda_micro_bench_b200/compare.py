"""Comparison rows of a results.json, as a Markdown table.

The reference's report carries one comparison row, DRAM bandwidth through
the load/store units against TMA (results/report.html:550-559,
TMA_LSU_COMPARE: memory_dram.read_bw_gibps against
tma.tma_g2s_load_bw_gibps).  This module renders that row and the rows the
B200 probes add beside it: the copy stream against the TMA tile copy, the
legacy mma.sync issue rate against the tcgen05 GEMM (bf16 and e4m3; in the
plain and the die-split tile order, and with bf16 C), and the NVLink ring and
all-to-all by peer stores, bulk copies and copy engines.  Each row names the
keys it reads; a key the run did not log shows as "n/a".

    python -m cuda_micro_bench_b200.compare [results/results.json]
"""

import argparse
import json
import sys
from pathlib import Path

# (row name, unit, [(label, section, key, scale to the row's unit)]); higher is better
# in every row.
ROWS = [
    ("DRAM read bandwidth", "GiB/s", [
        ("LSU stream read (fp32 sum)", "memory_dram", "read_bw_gibps", 1.0),
        ("TMA bulk tile load, read only", "tma", "tma_g2s_load_bw_gibps", 1.0)]),
    ("DRAM copy bandwidth (read + write)", "GB/s", [
        ("LSU copy stream", "memory_dram", "copy_bw_gbps", 1.0),
        ("TMA tile load + TMA store", "tma", "tile_copy_bw_gbps", 1.0)]),
    ("BF16 tensor throughput", "TFLOP/s", [
        ("mma.sync m16n8k16 issue rate (registers only)", "tensor_core_extended",
         "bf16_m16n8k16_throughput_TFs", 1.0),
        ("tcgen05 GEMM 8192^3, plain tile order", "tensor_core_tcgen05",
         "bf16_gemm_8192_plain_order_tflops", 1.0),
        ("tcgen05 GEMM 8192^3 (TMA, TMEM, checked; die-split order)", "tensor_core_tcgen05",
         "bf16_gemm_8192_tflops", 1.0),
        ("tcgen05 GEMM 8192^3, bf16 C", "tensor_core_tcgen05", "bf16_gemm_8192_bf16out_tflops",
         1.0)]),
    ("FP8 e4m3 tensor throughput", "TFLOP/s", [
        ("mma.sync m16n8k32 issue rate (registers only)", "tensor_core_extended",
         "fp8_m16n8k32_throughput_TFs", 1.0),
        ("tcgen05 GEMM 8192^3, plain tile order", "tensor_core_tcgen05",
         "fp8_e4m3_gemm_8192_plain_order_tflops", 1.0),
        ("tcgen05 GEMM 8192^3 (TMA, TMEM, checked; die-split order)", "tensor_core_tcgen05",
         "fp8_e4m3_gemm_8192_tflops", 1.0),
        ("tcgen05 GEMM 8192^3, bf16 C", "tensor_core_tcgen05",
         "fp8_e4m3_gemm_8192_bf16out_tflops", 1.0)]),
    ("NVLink ring, egress per GPU", "GB/s", [
        ("SM peer stores", "p2p", "ring_store_link_gbps", 1.0),
        ("SM bulk copies", "p2p", "ring_bulk_link_gbps", 1.0),
        ("copy engines", "p2p", "ring_copy_engine_link_gbps", 1.0)]),
    ("NVLink all-to-all, egress per GPU", "GB/s", [
        ("SM peer stores", "p2p", "alltoall_store_link_gbps", 1.0),
        ("SM bulk copies", "p2p", "alltoall_bulk_link_gbps", 1.0),
        ("copy engines", "p2p", "alltoall_copy_engine_link_gbps", 1.0)]),
]


def value(results, section, key):
    e = results.get(section, {}).get(key)
    if e is None or e.get("unit") == "N/A" or e.get("value") is None:
        return None
    return float(e["value"])


def rows(doc):
    """(row name, unit, [(label, value or None)], best label or None)."""
    results = doc.get("results", {})
    out = []
    for name, unit, cols in ROWS:
        vals = []
        for label, sec, key, scale in cols:
            v = value(results, sec, key)
            vals.append((label, None if v is None else v * scale))
        known = [(v, label) for label, v in vals if v is not None]
        best = max(known)[1] if len(known) > 1 else None
        out.append((name, unit, vals, best))
    return out


def markdown(doc):
    lines = [f"Comparison rows: {doc.get('device', '?')} ({doc.get('architecture', '?')}, "
             f"{doc.get('sm_count', '?')} SMs)", "",
             "| row | path | value | vs first path |", "|---|---|---|---|"]
    for name, unit, vals, best in rows(doc):
        first = vals[0][1]
        for i, (label, v) in enumerate(vals):
            shown = "n/a" if v is None else f"{v:,.1f} {unit}"
            ratio = ("" if i == 0 or v is None or not first else f"{v / first:.2f}x")
            mark = " (best)" if label == best else ""
            lines.append(f"| {name if i == 0 else ''} | {label}{mark} | {shown} | {ratio} |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("path", nargs="?", default="results/results.json")
    args = ap.parse_args(argv)
    sys.stdout.write(markdown(json.loads(Path(args.path).read_text())))
    return 0


if __name__ == "__main__":
    sys.exit(main())
