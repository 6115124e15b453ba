"""CPU tests of bench.py's contract parts that need no GPU: the reference
arm's JSON line and the argument checks."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    env = dict(os.environ, RANK="0", WORLD_SIZE="1")
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          capture_output=True, text=True, timeout=600, env=env)


def test_reference_arm_json_line():
    p = _run("--impl", "reference", "--steps", "2", "--warmup", "3")
    assert p.returncode == 0, p.stderr
    lines = [l for l in p.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "config", "impl",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["steps"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_exit_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2")
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--steps", "2", "--warmup", "3"],
                       capture_output=True, text=True, timeout=120, env=env)
    assert p.returncode == 0 and p.stdout.strip() == ""


def test_warmup_is_raised_to_three():
    p = _run("--impl", "reference", "--steps", "2", "--warmup", "1")
    assert p.returncode == 0, p.stderr
    assert json.loads(p.stdout.strip().splitlines()[-1])["warmup"] == 3
    assert "raised to 3" in p.stderr


def test_argument_checks():
    p = _run("--steps", "0")
    assert p.returncode != 0 and "--steps must be >= 1" in p.stderr
    p = _run("--gpus", "2")
    assert p.returncode != 0 and "torchrun" in p.stderr


def test_failed_checks_finds_every_failed_probe_flag():
    sys.path.insert(0, ROOT)
    import bench

    probes = {"stream_1gib": {"copy": {"bit_exact": True, "status": 0}},
              "gemm": {"bf16": {"within_1e-2": False, "status": 0},
                       "cublas_same_operands": {"bf16_TFLOP/s": 1500.0}},
              "tma_16384": {"tma_1d": {"landed_bytes_match": True, "status": 3}},
              "p2p_256mib": {"ring_store": {"bit_exact": False},
                             "nccl_reference": {"ring_nccl": {"received_first_chunk_ok": False}}},
              "chase_512mib": {"endpoint_matches_host_walk": True}}
    assert sorted(bench.failed_checks(probes)) == [
        "gemm.bf16.within_1e-2=False", "p2p_256mib.ring_store.bit_exact=False",
        "tma_16384.tma_1d.status=3"]
    assert bench.failed_checks({"a": {"bit_exact": True, "status": 0}}) == []
