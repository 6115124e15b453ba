"""GPU tests of the drop-in layer: the CLI's full run writes a results file
with every key the reference's report reads, the measured values are
physically plausible (the reference's validator checks, retargeted to B200:
tools/validate_results.py:56-77), and the legacy mma.sync probes keep their
constant-operand sums."""

import ctypes
import json
import math
import os
import subprocess

import numpy as np
import pytest

from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "cuda_micro_bench_b200", "bin", "cmb_b200")


def test_cli_full_run(cuda, tmp_path):
    out = tmp_path / "results.json"
    p = subprocess.run([EXE, "--json", f"--out={out}"], capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    doc = json.loads(out.read_text())
    assert doc["device"].startswith("NVIDIA B200") and doc["architecture"] == "10.0"
    res = doc["results"]
    keys = [tuple(l.split()) for l in open(os.path.join(ROOT, "tests", "golden", "report_keys.txt"))
            if l.strip()]
    for sec, key in keys:
        assert key in res[sec], (sec, key)
    v = lambda s, k: res[s][k]["value"]
    for sec, entries in res.items():
        for key, e in entries.items():
            if e["unit"] == "N/A":
                assert e["value"] is None
            else:
                assert isinstance(e["value"], (int, float)) and math.isfinite(e["value"]), (sec, key)
    assert 3000 < v("memory", "dram_read_bw_gbps") <= 8000 * 1.1
    assert 3000 < v("memory_dram", "copy_bw_gbps") <= 8000 * 1.1
    assert v("memory_dram", "copy_verified") == 1.0
    assert v("memory_dram", "chase_endpoint_verified") == 1.0
    assert v("memory_dram", "chase_working_set_bytes") == 512 * 2**20
    assert v("memory_dram", "chase_min_sector_footprint_bytes") > 126e6
    l1, l2, dram = (v("memory", f"{lvl}_latency_cyc") for lvl in ("l1", "l2", "dram"))
    assert 0 < l1 < l2 < dram, (l1, l2, dram)
    assert v("tma", "tma_1d_load_latency_cyc") > 0 and v("tma", "tma_g2s_load_bw_gibps") > 1000
    assert v("tma", "tile_copy_verified") == 1.0
    for p_ in ("bf16_gemm_8192", "fp8_e4m3_gemm_8192"):
        assert v("tensor_core_tcgen05", p_ + "_verified") == 1.0
        assert v("tensor_core_tcgen05", p_ + "_max_rel_err") <= 1e-2
    assert v("tensor_core_tcgen05", "bf16_gemm_8192_tflops") > 500
    assert v("tensor_core_tcgen05", "fp8_e4m3_gemm_8192_tflops") > 1000
    assert v("tensor_core_extended", "fp16_m16n8k16_latency_cycles") > 0
    assert v("tensor_core", "mma_m16n8k8_throughput_tflops") > 0
    assert v("memory_more", "l2_aggregate_verified") == 1.0
    assert v("memory_more", "l2_aggregate_bw_gbps") > v("memory", "dram_read_bw_gbps")
    assert 5 < v("pcie", "htod_bandwidth_GiB_s") < 128 and 5 < v("pcie", "dtoh_bandwidth_GiB_s") < 128
    # the host reference on the same data, and the seeds of the synthetic inputs
    assert v("host_ref", "cores") >= 1
    assert v("host_ref", "sum_gbps") > 0 and v("host_ref", "memcpy_gbps") > 0
    assert v("host_ref", "chase_ns_per_hop") > 1 and v("host_ref", "gemm_fp64_tiles_tflops") > 0
    assert v("memory_dram", "stream_seed") == 0x5EED and v("memory_dram", "chase_seed") == 0xC0DA
    assert v("tensor_core_tcgen05", "gemm_seed") == 0x6E33 and v("tma", "tile_seed") == 0x5EED
    # the die map the GEMMs ran with
    assert v("tensor_core_tcgen05", "sms_on_die0") + v("tensor_core_tcgen05", "sms_on_die1") == 148
    from cuda_micro_bench_b200 import compare, validate_results
    assert validate_results.check(doc) == []
    table = compare.markdown(doc)
    assert "tcgen05 GEMM" in table and "n/a" not in table.split("NVLink")[0]
    print(p.stdout)


def test_cli_single_section_writes_only_it(cuda, tmp_path):
    out = tmp_path / "results.json"
    p = subprocess.run([EXE, "--tma", f"--out={out}"], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    res = json.loads(out.read_text())["results"]
    assert set(res) == {"tma"}


@pytest.mark.parametrize("kind,k", [(0, 8), (2, 16), (3, 32), (4, 32)])
def test_mma_sync_constant_sums(cuda, cmb, kind, k):
    iters = 1000
    cyc = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    val = cuda.zeros(64, dtype=cuda.float64, device="cuda")
    cmb.check("cmb_mma_sync_latency", kind, iters, dptr(cyc), dptr(val), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert float(val[0]) == iters * k and int(cyc.item()) > 0
    cmb.check("cmb_mma_sync_throughput", kind, iters, 4, 8, dptr(val), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert bool((val[:32] == 4 * iters * k).all())


def test_compare_bytes(cuda, cmb):
    a = cuda.randint(0, 255, (1 << 20,), dtype=cuda.uint8, device="cuda")
    b = a.clone()
    m = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    cmb.check("cmb_compare_bytes", dptr(a), dptr(b), a.numel(), dptr(m), stream_handle(cuda))
    assert int(m.item()) == 0
    b[12345] ^= 1
    b[-1] ^= 1
    cmb.check("cmb_compare_bytes", dptr(a), dptr(b), a.numel(), dptr(m), stream_handle(cuda))
    assert int(m.item()) == 2
    cmb.check("cmb_compare_bytes", ctypes.c_void_p(a.data_ptr() + 1),
              ctypes.c_void_p(b.data_ptr() + 1), a.numel() - 1, dptr(m), stream_handle(cuda))
    assert int(m.item()) == 2
