"""GPU test of the drop-in: the reference's own executable (its main.cu,
result logger and out-of-scope sections, built from its sources by
oracle/Makefile target ref-dropin) with the probe sections taken from
libcmb_b200.so.  Run with the reference's flags, it must exit 0 and its own
JSON writer must write every report key of those sections
(results/report.html reads them), with the library's self-check keys set."""

import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(ROOT, "oracle", "_ref", "ref_dropin")

# Sections the library provides, and the keys of the reference's shared
# `memory` section that they log (the rest come from mem_shared.cu).
LIBRARY_SECTIONS = {"memory_dram", "memory_cache", "tma", "tensor_core", "tensor_core_extended"}
LIBRARY_MEMORY_KEYS = {"dram_read_bw_gbps", "dram_latency_cyc", "l1_latency_cyc", "l2_latency_cyc"}


@pytest.mark.skipif(not os.path.exists(DROPIN),
                    reason="oracle/_ref/ref_dropin is built only where the reference sources are")
def test_reference_main_runs_library_sections(cuda, tmp_path):
    (tmp_path / "results").mkdir()
    flags = ["--device", "--memory", "--cache", "--tma", "--tensor", "--tensor-ext"]
    p = subprocess.run([DROPIN, *flags], cwd=tmp_path, capture_output=True, text=True,
                       timeout=900)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    doc = json.loads((tmp_path / "results" / "results.json").read_text())
    # the device header arrives through the sink (the reference's own
    # device_info section sets it too)
    assert doc["device"].startswith("NVIDIA B200") and doc["architecture"] == "10.0"
    res = doc["results"]
    keys = [tuple(l.split()) for l in open(os.path.join(ROOT, "tests", "golden", "report_keys.txt"))
            if l.strip()]
    want = [(s, k) for s, k in keys
            if s in LIBRARY_SECTIONS or (s == "memory" and k in LIBRARY_MEMORY_KEYS)]
    assert len(want) >= 14
    for sec, key in want:
        assert key in res.get(sec, {}), (sec, key)
        assert res[sec][key]["value"] is not None, (sec, key)  # measured, not "N/A"
    # the reference's own device_info section ran beside the library's
    assert res["topology"]["sm_count"]["value"] == 148.0
    # the library's checks, logged through the sink
    for sec, key in [("memory_dram", "copy_verified"), ("memory_dram", "chase_endpoint_verified"),
                     ("tma", "tile_copy_verified"), ("tma", "tma_1d_verified"),
                     ("tensor_core_tcgen05", "bf16_gemm_8192_verified"),
                     ("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_verified")]:
        assert res[sec][key]["value"] == 1.0, (sec, key)
    assert 5000 < res["memory_dram"]["copy_bw_gbps"]["value"] < 9000
