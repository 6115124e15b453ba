"""CPU tests of the native library: it loads, exports every entry point the
header declares, writes results.json byte-identical to the reference's own
logger, and its host-side chase builder matches the oracle bit for bit.
No GPU call is made here."""

import ctypes
import os
import re

import numpy as np
import pytest

from oracle import ptr

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def declared_functions():
    names = []
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(inc, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(cmb_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ["cmb_stream_copy", "cmb_stream_sum_f32", "cmb_chase_run",
                 "cmb_results_write_json"]:
        assert must in names


def test_every_declared_symbol_is_exported(cmb):
    missing = [n for n in declared_functions() if not hasattr(cmb.lib, n)]
    assert not missing, missing


def test_every_declared_symbol_has_a_signature(cmb):
    from cuda_micro_bench_b200.capi import SIGNATURES
    missing = [n for n in declared_functions() if n not in SIGNATURES]
    assert not missing, missing


def test_status_strings(cmb):
    assert cmb.lib.cmb_status_string(0) == b"CMB_OK"
    assert cmb.lib.cmb_status_string(3) == b"CMB_ERR_TIMEOUT"
    assert cmb.lib.cmb_status_string(99) == b"CMB_ERR_UNKNOWN"


def _run_script(cmb, script_path, out_path):
    cmb.check("cmb_results_clear")
    for line in open(script_path).read().splitlines():
        f = line.split("\t")
        if f[0] == "D":
            cmb.check("cmb_results_set_device", f[1].encode(), f[2].encode(), int(f[3]),
                      int(f[4]), int(f[5]), int(f[6]))
        elif f[0] == "L":
            unit = f[4] if len(f) > 4 else ""
            cmb.check("cmb_results_log", f[1].encode(), f[2].encode(), float(f[3]), unit.encode())
    cmb.check("cmb_results_write_json", str(out_path).encode())


@pytest.mark.parametrize("name", ["memory", "edge", "empty"])
def test_results_json_matches_reference_logger(cmb, tmp_path, name):
    out = tmp_path / "results.json"
    _run_script(cmb, os.path.join(GOLDEN, f"logger_{name}.script"), out)
    golden = open(os.path.join(GOLDEN, f"logger_{name}.json"), "rb").read()
    assert out.read_bytes() == golden


def test_results_json_unwritable_path(cmb, tmp_path):
    rc = cmb.lib.cmb_results_write_json(str(tmp_path / "no" / "such" / "dir.json").encode())
    assert rc == 6  # CMB_ERR_IO
    assert b"Cannot open results path" in cmb.lib.cmb_last_error()


@pytest.mark.parametrize("slots,seed", [(1, 0), (7, 1), (4096, 2), (1 << 16, 0xC0DA)])
def test_chase_builder_matches_oracle(cmb, orc, slots, seed):
    mine = np.empty(slots * 32, np.uint32)
    ref = np.empty_like(mine)
    cmb.check("cmb_chase_build_links", ctypes.c_void_p(mine.ctypes.data), mine.nbytes,
              ctypes.c_uint64(seed))
    orc.orc_chase_build(ptr(ref), ref.nbytes, seed)
    assert np.array_equal(mine, ref)
    assert orc.orc_chase_is_single_cycle(ptr(mine), mine.nbytes) == 1


def test_chase_builder_rejects_bad_sizes(cmb):
    buf = np.empty(64, np.uint32)
    assert cmb.lib.cmb_chase_build_links(ctypes.c_void_p(buf.ctypes.data), 100, 0) == 1
    assert cmb.lib.cmb_chase_build_links(None, 128, 0) == 1


def test_chase_host_walk_matches_oracle(cmb, orc):
    links = np.empty(1000 * 32, np.uint32)
    orc.orc_chase_build(ptr(links), links.nbytes, 3)
    out = ctypes.c_uint32(0)
    for hops in (0, 1, 999, 1000, 12345):
        cmb.check("cmb_chase_host_walk", ctypes.c_void_p(links.ctypes.data), links.size,
                  ctypes.c_uint64(hops), ctypes.byref(out))
        assert out.value == orc.orc_chase_walk(ptr(links), hops, 0)
    links[0] = 1 << 30  # leaves the array on the first hop
    assert cmb.lib.cmb_chase_host_walk(ctypes.c_void_p(links.ctypes.data), links.size, 5,
                                       ctypes.byref(out)) == 1


def _report_keys():
    return [tuple(l.split()) for l in open(os.path.join(GOLDEN, "report_keys.txt")) if l.strip()]


def test_report_placeholders_cover_every_report_key(cmb, tmp_path):
    import json

    cmb.check("cmb_results_clear")
    cmb.check("cmb_results_set_device", b"NVIDIA B200", b"10.0", 148, 1965000, 3996000, 8192)
    cmb.check("cmb_results_log", b"memory", b"dram_latency_cyc", 812.0, b"cycles")
    cmb.check("cmb_results_log_report_placeholders")
    out = tmp_path / "r.json"
    cmb.check("cmb_results_write_json", str(out).encode())
    data = json.loads(out.read_text())["results"]
    keys = _report_keys()
    assert len(keys) == 195
    for sec, key in keys:
        assert key in data[sec], (sec, key)
    # measured values are kept, the rest are null with unit N/A
    assert data["memory"]["dram_latency_cyc"]["value"] == 812.0
    assert data["atomics"]["block_reduce_latency_cyc"] == {"value": None, "unit": "N/A"}


def test_cli_usage_and_unknown_flag(tmp_path):
    import subprocess

    exe = os.path.join(ROOT, "cuda_micro_bench_b200", "bin", "cmb_b200")
    out = tmp_path / "x.json"
    p = subprocess.run([exe, "--help", f"--out={out}"], capture_output=True, text=True)
    assert p.returncode == 0 and "--memory" in p.stdout and "--tensor-ext" in p.stdout
    assert not out.exists()  # no section ran, nothing to write
    p = subprocess.run([exe, "--bogus", f"--out={out}"], capture_output=True, text=True)
    assert p.returncode == 1 and "Unknown option: --bogus" in p.stdout
    assert not out.exists()


def test_die_map_entry_points_reject_bad_arguments(cmb):
    """Argument checks that come before any device call (no GPU needed)."""

    def rc(fn, *args):
        return getattr(cmb.lib, fn)(*args)

    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    two_dies = np.array([0, 0, 1, 1, 0xFF, 1], np.uint8)
    assert rc("cmb_gemm_set_sm_die_map", p(two_dies), 300) == 1  # more ids than a map holds
    assert rc("cmb_gemm_set_sm_die_map", p(two_dies), -1) == 1
    bad_label = np.array([0, 1, 2, 1], np.uint8)
    assert rc("cmb_gemm_set_sm_die_map", p(bad_label), 4) == 1
    assert "not 0 or 1" in cmb.lib.cmb_last_error().decode()
    one_die = np.array([0, 0, 0xFF, 0], np.uint8)
    assert rc("cmb_gemm_set_sm_die_map", p(one_die), 4) == 1
    assert "both dies" in cmb.lib.cmb_last_error().decode()
    out = np.zeros(256, np.uint8)
    n = ctypes.c_int(0)
    assert rc("cmb_sm_die_map", None, 256, ctypes.byref(n), None, None) == 1
    assert rc("cmb_sm_die_map", p(out), 256, None, None, None) == 1
    assert rc("cmb_sm_die_map", p(out), 0, ctypes.byref(n), None, None) == 1
