"""GPU test of bench.py's JSON-line contract on a short run: every key the
driver reads is present and consistent (roofline, e2e, clocks, launches,
CPU baseline), and the probe-only mode reports checked results."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, timeout=600):
    env = dict(os.environ, RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                       capture_output=True, text=True, timeout=timeout, env=env)
    assert p.returncode == 0, p.stderr[-3000:]
    lines = [l for l in p.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, p.stdout
    return json.loads(lines[0])


def test_headline_line_contract():
    d = _bench("--steps", "5", "--warmup", "3", "--gib", "1", "--no-probes", "--e2e-steps", "1")
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "roofline",
              "e2e", "gpu_launches", "clocks", "cpu_baseline"):
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 5 and d["warmup"] == 3 and d["unit"] == "GB/s"
    assert d["gpu_launches"] == 5
    rf = d["roofline"]
    assert rf["bound"] == "hbm" and rf["unit"] == "GB/s"
    assert abs(rf["frac"] - rf["achieved"] / rf["peak"]) < 1e-3
    assert 0.5 < rf["frac"] < 1.2  # a working copy stream on a B200
    e = d["e2e"]
    assert e["h2d_bytes_per_step"] == e["d2h_bytes_per_step"] == 1 << 30
    assert 0 < e["value"] < d["value"]  # PCIe-bound, below the in-HBM rate
    assert "sm_mhz" in d["clocks"] and "reasons" in d["clocks"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] > 0


def test_probe_only_mode_checks_results():
    d = _bench("--probe", "stream", "--probe", "tma")["probes"]
    assert d["copy_1gib"]["bit_exact"] and d["sum_1gib"]["within_1e-5"]
    for k in ("tile_copy_4stage", "tile_copy_3stage", "tile_copy_tma_load_lsu_store"):
        assert d["tma_16384"][k]["bit_exact"] and d["tma_16384"][k]["status"] == 0
