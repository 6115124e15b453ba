"""CPU tests of the drop-in boundary with the reference's own executable.

The reference's main.cu declares and calls `void cmb::benchmark_<section>()`
(src/main.cu:9-32) and writes `cmb::g_results` (src/result_logger.cu:8).
libcmb_b200.so must therefore export exactly the C ABI plus those section
entry points, and keep its own results table private, so a reference build
that links it has one g_results (its own) that the library logs into
through cmb_results_set_sink().  No GPU is needed (on a machine with one,
the last test runs the global-memory section in a child process)."""

import ctypes
import os
import re
import shutil
import subprocess
import sys

import pytest

from tests.test_capi import declared_functions

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(ROOT, "oracle", "_ref", "ref_dropin")

REFERENCE_SECTIONS = ["global_memory", "cache", "tma", "tensor_core", "tensor_core_extended"]
EXPORTED_CXX = {f"cmb::benchmark_{s}()" for s in REFERENCE_SECTIONS + ["multi_gpu"]}


def _dynamic_symbols(path, defined=True):
    args = ["nm", "-D", "-C"] + (["--defined-only"] if defined else ["--undefined-only"])
    out = subprocess.run(args + [path], capture_output=True, text=True, check=True).stdout
    names = []
    for line in out.splitlines():
        parts = line.split(None, 2)
        if len(parts) >= 2:
            names.append(parts[-1].split("@")[0])
    return names


needs_nm = pytest.mark.skipif(shutil.which("nm") is None, reason="binutils nm not installed")


@needs_nm
def test_library_exports_only_c_abi_and_reference_sections(cmb):
    names = _dynamic_symbols(cmb.library_path)
    c_names = {n for n in names if n.startswith("cmb_")}
    cxx = {n for n in names if not n.startswith("cmb_")}
    assert cxx == EXPORTED_CXX, sorted(cxx ^ EXPORTED_CXX)
    assert c_names == set(declared_functions()), sorted(c_names ^ set(declared_functions()))
    assert not any("g_results" in n or "ResultLogger" in n for n in names)


def test_results_sink_forwards_every_entry(cmb):
    log_t = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_double,
                             ctypes.c_char_p, ctypes.c_void_p)
    dev_t = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                             ctypes.c_int, ctypes.c_int, ctypes.c_void_p)
    logged, devices = [], []
    on_log = log_t(lambda s, k, v, u, _: logged.append((s.decode(), k.decode(), v, u.decode())))
    on_dev = dev_t(lambda n, a, sm, c, m, b, _: devices.append((n.decode(), a.decode(), sm, c, m, b)))
    try:
        cmb.check("cmb_results_clear")
        cmb.check("cmb_results_set_sink", ctypes.cast(on_log, ctypes.c_void_p),
                  ctypes.cast(on_dev, ctypes.c_void_p), None)
        cmb.check("cmb_results_set_device", b"NVIDIA B200", b"10.0", 148, 1965000, 3996000, 7680)
        cmb.check("cmb_results_log", b"memory_dram", b"copy_bw_gbps", 6673.5, b"GB/s")
        cmb.check("cmb_results_log", b"tma", b"tma_1d_load_latency_cyc", 0.0, b"N/A")
        assert devices == [("NVIDIA B200", "10.0", 148, 1965000, 3996000, 7680)]
        assert logged == [("memory_dram", "copy_bw_gbps", 6673.5, "GB/s"),
                          ("tma", "tma_1d_load_latency_cyc", 0.0, "N/A")]
        cmb.check("cmb_results_set_sink", None, None, None)  # uninstall
        cmb.check("cmb_results_log", b"memory_dram", b"read_bw_gibps", 1.0, b"GiB/s")
        assert len(logged) == 2
    finally:
        cmb.check("cmb_results_set_sink", None, None, None)
        cmb.check("cmb_results_clear")


@needs_nm
@pytest.mark.skipif(not os.path.exists(DROPIN),
                    reason="oracle/_ref/ref_dropin is built only where the reference sources are")
def test_reference_executable_takes_probe_sections_from_library():
    """The reference's main.cu, linked by oracle/Makefile target ref-dropin,
    defines its own g_results and leaves exactly the five probe sections to
    the library."""
    undefined = _dynamic_symbols(DROPIN, defined=False)
    for s in REFERENCE_SECTIONS:
        assert f"cmb::benchmark_{s}()" in undefined, s
    assert "cmb_results_set_sink" in undefined
    local = subprocess.run(["nm", "-C", DROPIN], capture_output=True, text=True,
                           check=True).stdout
    assert re.search(r" B cmb::g_results$", local, re.M)
    for s in ["device_info", "memory_more", "pcie", "shared_memory"]:  # the reference's own
        assert re.search(rf" T cmb::benchmark_{s}\(\)$", local, re.M), s
    dyn = subprocess.run(["readelf", "-d", DROPIN], capture_output=True, text=True).stdout
    assert "libcmb_b200.so" in dyn and "$ORIGIN/../../cuda_micro_bench_b200/lib" in dyn


def test_reference_entry_points_exit_like_the_reference(cmb):
    """`void cmb::benchmark_global_memory()` keeps the reference's error
    behaviour (CUDA_CHECK, include/utils.h:11-19): a failure prints the reason
    and ends the process with EXIT_FAILURE.  Without a GPU the device query
    fails; on a machine with a B200 the section runs and returns."""
    script = (
        "import ctypes, sys\n"
        "lib = ctypes.CDLL(sys.argv[1])\n"
        "getattr(lib, '_ZN3cmb23benchmark_global_memoryEv')()\n"
        "print('returned')\n")
    r = subprocess.run([sys.executable, "-c", script, cmb.library_path], capture_output=True,
                       text=True, timeout=600)
    if r.returncode == 0:
        assert "returned" in r.stdout
    else:
        assert r.returncode == 1, (r.returncode, r.stderr)
        assert "benchmark_global_memory failed: CMB_ERR_CUDA" in r.stderr, r.stderr
        assert "returned" not in r.stdout
