"""Checks a results.json written by cmb_b200 (or by cmb_results_write_json)
for full-run coverage of the report's keys, units, finite values and the
physical limits of a B200.

The reference's tools/validate_results.py does the same for the GPU it was
written on (device identity asserts at :42-49, coverage :50-51, units and
finite values :53-65, physical sanity :67-93).  This restatement keeps those
rules, takes the device identity, bounds and key list from the B200 (the key
list from the library's own table of the report's paths,
cmb_report_key_count / cmb_report_key) and adds the checks of the probes the
reference does not have: verified copies, chase endpoints, tiles and GEMMs,
tensor-core and NVLink ceilings.

    python -m cuda_micro_bench_b200.validate_results [results/results.json] [--partial]

Exit status 0 when every check passes, 1 otherwise (each failure printed).
"""

import argparse
import ctypes
import json
import math
import sys
from pathlib import Path

# B200 nominal limits; measured values may exceed a copy-based peak a little,
# never these by more than the stated headroom.
B200 = {
    "name_prefix": "NVIDIA B200",
    "architecture": "10.0",
    "sm_count": 148,
    "hbm_gbs": 8000.0,          # HBM3e, DGX figure (7.7 TB/s HGX)
    "l2_bytes": 126e6,          # 126 MB
    "bf16_tflops": 2250.0,      # dense
    "fp8_tflops": 4500.0,       # dense
    "nvlink_gbs": 900.0,        # per direction per GPU
    "pcie_gibs": 64.0,          # Gen5 x16, either direction
}
HEADROOM = 1.10
GIB_PER_GB = 1e9 / 2**30


def report_keys():
    """(section, key) paths the reference's report reads, from the library."""
    from cuda_micro_bench_b200 import lib

    keys = []
    sec, key = ctypes.c_char_p(), ctypes.c_char_p()
    for i in range(lib.cmb_report_key_count()):
        if lib.cmb_report_key(i, ctypes.byref(sec), ctypes.byref(key)) != 0:
            raise RuntimeError(f"cmb_report_key({i}) failed")
        keys.append((sec.value.decode(), key.value.decode()))
    return keys


def check(doc, full=True, keys=None):
    """Returns the list of failed checks (empty when the document passes).
    full=False skips the coverage checks (a run of selected sections)."""
    problems = []
    results = doc.get("results", {})

    def fail(msg):
        problems.append(msg)

    def val(section, key):
        e = results.get(section, {}).get(key)
        if e is None or e.get("unit") == "N/A":
            return None
        return e.get("value")

    def bound(section, key, lo, hi, what):
        v = val(section, key)
        if v is not None and not (lo < v <= hi):
            fail(f"{section}.{key} = {v} outside ({lo}, {hi}]: {what}")

    def flag(section, key):
        v = val(section, key)
        if v is not None and v != 1.0:
            fail(f"{section}.{key} = {v}: the probe's output check failed")

    # device identity
    if not str(doc.get("device", "")).startswith(B200["name_prefix"]):
        fail(f"device {doc.get('device')!r} is not a B200")
    if doc.get("architecture") != B200["architecture"]:
        fail(f"architecture {doc.get('architecture')!r} is not {B200['architecture']}")
    if doc.get("sm_count") != B200["sm_count"]:
        fail(f"sm_count {doc.get('sm_count')} is not {B200['sm_count']}")

    # coverage
    if full:
        for section, key in (keys if keys is not None else report_keys()):
            if key not in results.get(section, {}):
                fail(f"missing report metric {section}.{key}")

    # units and values
    for section, metrics in results.items():
        for key, e in metrics.items():
            v, unit = e.get("value"), e.get("unit")
            if unit == "N/A":
                if v is not None:
                    fail(f"{section}.{key}: unit N/A with value {v}")
                continue
            if not isinstance(v, (int, float)) or isinstance(v, bool) or not math.isfinite(v):
                fail(f"{section}.{key}: value {v!r} is not a finite number")
            elif v < 0:
                fail(f"{section}.{key}: negative value {v}")

    # memory
    hbm = B200["hbm_gbs"] * HEADROOM
    bound("memory", "dram_read_bw_gbps", 0, hbm, "HBM3e read bandwidth")
    bound("memory_dram", "copy_bw_gbps", 0, hbm, "HBM3e copy bandwidth")
    bound("memory_dram", "read_bw_gibps", 0, hbm * GIB_PER_GB, "HBM3e read bandwidth")
    bound("memory_dram", "copy_max_bw_gibps", 0, hbm * GIB_PER_GB, "HBM3e copy bandwidth")
    flag("memory_dram", "copy_verified")
    flag("memory_dram", "chase_endpoint_verified")
    ws = val("memory_dram", "chase_working_set_bytes")
    if ws is not None:
        if ws <= B200["l2_bytes"]:
            fail(f"memory_dram.chase_working_set_bytes = {ws} fits in L2: not a DRAM latency")
        # every 128-byte slot is one link of a single cycle; a sample walks
        # whole laps of it (the reference one lap, this build four)
        loads, slots = val("memory_dram", "chase_loads_per_sample"), ws / 128
        if loads is not None and (loads < slots or loads % slots != 0):
            fail(f"memory_dram.chase_loads_per_sample = {loads}: not whole laps of the "
                 f"{slots:.0f}-slot cycle (one link per 128-byte slot)")
    fp = val("memory_dram", "chase_min_sector_footprint_bytes")
    if fp is not None and fp <= B200["l2_bytes"]:
        fail(f"memory_dram.chase_min_sector_footprint_bytes = {fp} fits in L2")
    sw = val("memory_dram", "stream_working_set_bytes")
    if sw is not None and sw <= 2 * B200["l2_bytes"]:
        fail(f"memory_dram.stream_working_set_bytes = {sw}: under twice the L2")
    l2ws = val("memory_cache", "l2_chase_working_set_bytes")
    if l2ws is not None and l2ws >= B200["l2_bytes"]:
        fail(f"memory_cache.l2_chase_working_set_bytes = {l2ws} does not fit in L2")
    lat = [val("memory", f"{lvl}_latency_cyc") for lvl in ("l1", "l2", "dram")]
    if all(x is not None for x in lat) and not (0 < lat[0] < lat[1] < lat[2]):
        fail(f"latency order l1 < l2 < dram broken: {lat}")
    l2bw, dram = val("memory_more", "l2_aggregate_bw_gbps"), val("memory", "dram_read_bw_gbps")
    if l2bw is not None and dram is not None and l2bw <= dram:
        fail(f"memory_more.l2_aggregate_bw_gbps = {l2bw} not above the DRAM read {dram}")
    flag("memory_more", "l2_aggregate_verified")

    # TMA
    bound("tma", "tma_g2s_load_bw_gibps", 0, hbm * GIB_PER_GB, "TMA loads stream from HBM")
    bound("tma", "tile_copy_bw_gbps", 0, hbm, "TMA tile copy reads and writes HBM")
    bound("tma", "tma_1d_load_latency_cyc", 0, 1e6, "one 16-byte TMA round trip")
    flag("tma", "tile_copy_verified")

    # tensor cores
    for p, spec in (("bf16_gemm_8192", B200["bf16_tflops"]),
                    ("fp8_e4m3_gemm_8192", B200["fp8_tflops"])):
        bound("tensor_core_tcgen05", p + "_tflops", 0, spec * 1.05, "dense tensor peak")
        bound("tensor_core_tcgen05", p + "_bf16out_tflops", 0, spec * 1.05, "dense tensor peak")
        bound("tensor_core_tcgen05", p + "_plain_order_tflops", 0, spec * 1.05, "dense tensor peak")
        flag("tensor_core_tcgen05", p + "_verified")
        flag("tensor_core_tcgen05", p + "_bf16out_verified")
        err = val("tensor_core_tcgen05", p + "_max_rel_err")
        if err is not None and err > 1e-2:
            fail(f"tensor_core_tcgen05.{p}_max_rel_err = {err} above 1e-2")
    bound("peak", "fp16_tensor_tflops", 0, B200["bf16_tflops"] * 1.05, "dense fp16 tensor peak")
    # the host reference beside the GPU probes
    bound("host_ref", "cores", 0, 1024, "host threads")
    for k in ("sum_gbps", "memcpy_gbps", "chase_ns_per_hop", "gemm_fp64_tiles_tflops"):
        bound("host_ref", k, 0, 1e6, "a positive host timing")
    # the die map: every SM on one of two dies, far loads slower than near
    dies = [val("tensor_core_tcgen05", f"sms_on_die{d}") for d in (0, 1)]
    if all(x is not None for x in dies) and (min(dies) <= 0 or sum(dies) != B200["sm_count"]):
        fail(f"tensor_core_tcgen05.sms_on_die0/1 = {dies[0]} / {dies[1]}: not a split of "
             f"{B200['sm_count']} SMs")
    near = val("tensor_core_tcgen05", "die_near_load_latency_cyc")
    far = val("tensor_core_tcgen05", "die_far_load_latency_cyc")
    if near is not None and far is not None and not (0 < near < far):
        fail(f"tensor_core_tcgen05 die load latency near {near} / far {far} cycles")

    # host link and NVLink
    for k in ("htod_bandwidth_GiB_s", "dtoh_bandwidth_GiB_s"):
        bound("pcie", k, 0, B200["pcie_gibs"], "PCIe Gen5 x16")
    for key in results.get("p2p", {}):
        if key.endswith("_link_gbps"):
            bound("p2p", key, 0, B200["nvlink_gbs"] * 1.02, "NVLink 5 per direction")
        elif key.endswith("_verified"):
            flag("p2p", key)
    gpus = val("p2p", "gpus_used")
    agg = val("p2p", "sharded_stream_aggregate_gbps")
    if gpus and agg is not None and agg > gpus * hbm:
        fail(f"p2p.sharded_stream_aggregate_gbps = {agg} above {gpus} x HBM")
    return problems


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("path", nargs="?", default="results/results.json")
    ap.add_argument("--partial", action="store_true",
                    help="a run of selected sections: skip the report-coverage checks")
    args = ap.parse_args(argv)
    doc = json.loads(Path(args.path).read_text())
    problems = check(doc, full=not args.partial)
    n = sum(len(m) for m in doc.get("results", {}).values())
    if problems:
        for p in problems:
            print("FAIL", p)
        print(f"{args.path}: {len(problems)} failed checks over {n} metrics")
        return 1
    print(f"{args.path}: B200 result passes coverage, units, finite-value and physical-sanity "
          f"checks ({n} metrics)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
