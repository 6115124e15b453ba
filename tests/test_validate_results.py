"""CPU tests of the B200 results validator (the reference's
tools/validate_results.py restated for a B200): the key table it reads from
the library is the report's, a plausible full run passes, and each class of
broken document is caught."""

import copy
import json
import os

import pytest

from cuda_micro_bench_b200 import validate_results as vr

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _golden_keys():
    with open(os.path.join(ROOT, "tests", "golden", "report_keys.txt")) as f:
        return [tuple(line.split()) for line in f if line.strip()]


def test_library_key_table_is_the_reports():
    assert vr.report_keys() == _golden_keys()


def test_report_key_index_past_the_end(cmb):
    import ctypes
    a, b = ctypes.c_char_p(), ctypes.c_char_p()
    n = cmb.lib.cmb_report_key_count()
    assert cmb.lib.cmb_report_key(n, ctypes.byref(a), ctypes.byref(b)) == 1
    assert cmb.lib.cmb_report_key(0, None, None) == 1


# A full B200 run's measured keys with values in the ranges seen on the
# pool's GPUs (the rest are the report's "N/A" placeholders).
MEASURED = [
    ("memory", "dram_read_bw_gbps", 6470.0, "GB/s"),
    ("memory", "dram_latency_cyc", 846.0, "cycles"),
    ("memory", "l1_latency_cyc", 33.0, "cycles"),
    ("memory", "l2_latency_cyc", 480.0, "cycles"),
    ("memory_dram", "read_bw_gibps", 6025.0, "GiB/s"),
    ("memory_dram", "copy_max_bw_gibps", 6070.0, "GiB/s"),
    ("memory_dram", "copy_bw_gbps", 6520.0, "GB/s"),
    ("memory_dram", "copy_verified", 1.0, "bool"),
    ("memory_dram", "chase_endpoint_verified", 1.0, "bool"),
    ("memory_dram", "chase_working_set_bytes", 512.0 * 2**20, "bytes"),
    ("memory_dram", "chase_loads_per_sample", 4 * 512.0 * 2**20 / 128, "loads"),
    ("memory_dram", "chase_min_sector_footprint_bytes", 128.0 * 2**20, "bytes"),
    ("memory_dram", "stream_working_set_bytes", 2.0**30, "bytes"),
    ("memory_cache", "l2_chase_working_set_bytes", 64.0 * 2**20, "bytes"),
    ("memory_more", "l2_aggregate_bw_gbps", 12700.0, "GB/s"),
    ("memory_more", "l2_aggregate_verified", 1.0, "bool"),
    ("tma", "tma_1d_load_latency_cyc", 339.0, "cycles"),
    ("tma", "tma_g2s_load_bw_gibps", 6020.0, "GiB/s"),
    ("tma", "tile_copy_bw_gbps", 6100.0, "GB/s"),
    ("tma", "tile_copy_verified", 1.0, "bool"),
    ("tensor_core_tcgen05", "bf16_gemm_8192_tflops", 1519.0, "TFLOP/s"),
    ("tensor_core_tcgen05", "bf16_gemm_8192_plain_order_tflops", 1501.0, "TFLOP/s"),
    ("tensor_core_tcgen05", "sms_on_die0", 70.0, "count"),
    ("tensor_core_tcgen05", "gemm_seed", 28211.0, "seed"),
    ("memory_dram", "stream_seed", 24301.0, "seed"),
    ("host_ref", "cores", 16.0, "threads"),
    ("host_ref", "sum_gbps", 80.0, "GB/s"),
    ("host_ref", "memcpy_gbps", 120.0, "GB/s"),
    ("host_ref", "chase_ns_per_hop", 100.0, "ns"),
    ("host_ref", "gemm_fp64_tiles_tflops", 0.05, "TFLOP/s"),
    ("tensor_core_tcgen05", "sms_on_die1", 78.0, "count"),
    ("tensor_core_tcgen05", "die_near_load_latency_cyc", 610.0, "cycles"),
    ("tensor_core_tcgen05", "die_far_load_latency_cyc", 1000.0, "cycles"),
    ("tensor_core_tcgen05", "bf16_gemm_8192_verified", 1.0, "bool"),
    ("tensor_core_tcgen05", "bf16_gemm_8192_max_rel_err", 1.2e-5, ""),
    ("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_tflops", 2789.0, "TFLOP/s"),
    ("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_verified", 1.0, "bool"),
    ("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_max_rel_err", 1.2e-6, ""),
    ("peak", "fp16_tensor_tflops", 1519.0, "TFLOP/s"),
    ("pcie", "htod_bandwidth_GiB_s", 52.0, "GiB/s"),
    ("pcie", "dtoh_bandwidth_GiB_s", 52.5, "GiB/s"),
    ("p2p", "ring_store_link_gbps", 680.0, "GB/s"),
    ("p2p", "ring_store_verified", 1.0, "bool"),
    ("p2p", "gpus_used", 2.0, "GPUs"),
    ("p2p", "sharded_stream_aggregate_gbps", 13000.0, "GB/s"),
]


@pytest.fixture()
def full_doc(cmb, tmp_path):
    lib = cmb.lib
    lib.cmb_results_clear()
    try:
        assert lib.cmb_results_set_device(b"NVIDIA B200", b"10.0", 148, 1965000, 3996000, 8192) == 0
        for sec, key, v, unit in MEASURED:
            assert lib.cmb_results_log(sec.encode(), key.encode(), v, unit.encode()) == 0
        assert lib.cmb_results_log_report_placeholders() == 0
        path = tmp_path / "results.json"
        assert lib.cmb_results_write_json(str(path).encode()) == 0
    finally:
        lib.cmb_results_clear()
    return json.loads(path.read_text())


def test_plausible_full_run_passes(full_doc):
    assert vr.check(full_doc) == []


def _set(doc, sec, key, value, unit=None):
    d = copy.deepcopy(doc)
    e = d["results"].setdefault(sec, {}).setdefault(key, {"value": None, "unit": "N/A"})
    e["value"] = value
    if unit is not None:
        e["unit"] = unit
    return d


@pytest.mark.parametrize("sec,key,value,unit,needle", [
    ("memory_dram", "copy_bw_gbps", 9500.0, None, "HBM3e copy"),
    ("memory", "dram_read_bw_gbps", 0.0, None, "HBM3e read"),
    ("memory_dram", "chase_working_set_bytes", 64.0 * 2**20, None, "fits in L2"),
    ("memory_dram", "chase_loads_per_sample", 1000.0, None, "128-byte slot"),
    ("memory_dram", "chase_loads_per_sample", 1.5 * 512 * 2**20 / 128, None, "whole laps"),
    ("memory", "l2_latency_cyc", 20.0, None, "latency order"),
    ("memory_more", "l2_aggregate_bw_gbps", 6000.0, None, "not above the DRAM"),
    ("tma", "tile_copy_verified", 0.0, None, "output check failed"),
    ("tensor_core_tcgen05", "bf16_gemm_8192_tflops", 2500.0, None, "dense tensor peak"),
    ("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_max_rel_err", 0.05, None, "above 1e-2"),
    ("tensor_core_tcgen05", "bf16_gemm_8192_plain_order_tflops", 2600.0, None, "dense tensor peak"),
    ("tensor_core_tcgen05", "sms_on_die1", 70.0, None, "not a split of"),
    ("tensor_core_tcgen05", "die_far_load_latency_cyc", 500.0, None, "die load latency"),
    ("host_ref", "cores", 0.0, None, "host threads"),
    ("p2p", "ring_store_link_gbps", 1000.0, None, "NVLink 5"),
    ("pcie", "htod_bandwidth_GiB_s", 80.0, None, "PCIe Gen5"),
    ("atomics", "block_reduce_latency_cyc", 5.0, "N/A", "unit N/A with value"),
    ("memory", "dram_latency_cyc", float("nan"), None, "finite"),
    ("memory", "dram_latency_cyc", -1.0, None, "negative"),
])
def test_broken_documents_are_caught(full_doc, sec, key, value, unit, needle):
    problems = vr.check(_set(full_doc, sec, key, value, unit))
    assert any(needle in p for p in problems), problems


def test_device_identity_and_coverage(full_doc):
    d = copy.deepcopy(full_doc)
    d["device"] = "NVIDIA H100 80GB HBM3"
    d["architecture"] = "9.0"
    problems = vr.check(d)
    assert any("not a B200" in p for p in problems)
    assert any("architecture" in p for p in problems)
    d = copy.deepcopy(full_doc)
    del d["results"]["tma"]["tma_g2s_load_bw_gibps"]
    assert any("missing report metric tma.tma_g2s_load_bw_gibps" in p for p in vr.check(d))
    assert vr.check(d, full=False) == []


def test_cli_exit_status(full_doc, tmp_path, capsys):
    good = tmp_path / "good.json"
    good.write_text(json.dumps(full_doc))
    assert vr.main([str(good)]) == 0
    assert "passes" in capsys.readouterr().out
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps(_set(full_doc, "memory_dram", "copy_verified", 0.0)))
    assert vr.main([str(bad)]) == 1
    assert "FAIL memory_dram.copy_verified" in capsys.readouterr().out
