"""GPU test of cmb_stream_sum_f32_noalloc, the read-stream sum for callers
that cannot allocate device memory (their device memory is owned by another
allocator, or they cannot afford cudaMalloc/cudaFree on the path).  It must
give the same sum as cmb_stream_sum_f32, which uses a caller-allocated
workspace, on two calls in a row: the second call reuses the library's
static scratch left over from the first.  Further cases: an empty input,
inputs that start 1-3 floats past a 32-byte boundary (the 16-byte vector
kernel and the unaligned head), one call per GPU where there are several,
and a call after the device was reset (the scratch array is reloaded and
may move).

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.  It passes alone in a fresh
process and after the other tests."""

import ctypes
import json
import subprocess
import sys

import numpy as np
import pytest

from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu

REL_TOL_SUM = 1e-5  # the stream sum's stated tolerance


def _sum_with_workspace(cuda, cmb, x, n):
    ws_bytes = cmb.lib.cmb_stream_sum_workspace_bytes(n)
    ws = cuda.empty(ws_bytes, dtype=cuda.uint8, device="cuda")
    out = cuda.full((1,), float("nan"), dtype=cuda.float64, device="cuda")
    cmb.check("cmb_stream_sum_f32", dptr(x), n, dptr(out), dptr(ws), ws_bytes, stream_handle(cuda))
    return float(out.item())


def _sum_noalloc(cuda, cmb, x, n):
    out = cuda.full((1,), float("nan"), dtype=cuda.float64, device="cuda")
    cmb.check("cmb_stream_sum_f32_noalloc", dptr(x), n, dptr(out), stream_handle(cuda))
    return float(out.item())


def _check_equal(got, ref, n):
    assert np.isfinite(got)
    assert abs(got - ref) <= REL_TOL_SUM * max(abs(ref), 1e-30), (n, got, ref)
    # same kernel and launch shape: the sums agree exactly
    assert got == ref, (n, got, ref)


def test_noalloc_sum_matches_workspace_sum_twice(cuda, cmb):
    assert cmb.lib.cmb_stream_sum_noalloc_max_ctas() == 4096
    cases = [((1 << 26) + 3, 101), ((1 << 20) + 17, 202)]  # two calls in a row
    for n, seed in cases:
        x = cuda.empty(n, dtype=cuda.float32, device="cuda")
        cmb.check("cmb_fill_uniform_f32", dptr(x), n, ctypes.c_uint64(seed), stream_handle(cuda))
        _check_equal(_sum_noalloc(cuda, cmb, x, n), _sum_with_workspace(cuda, cmb, x, n), n)


def test_noalloc_sum_empty_input(cuda, cmb):
    x = cuda.zeros(4, dtype=cuda.float32, device="cuda")
    assert _sum_noalloc(cuda, cmb, x, 0) == 0.0
    assert _sum_with_workspace(cuda, cmb, x, 0) == 0.0


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_noalloc_sum_unaligned_start(cuda, cmb, offset):
    n = (1 << 22) + 5
    base = cuda.empty(n + 8, dtype=cuda.float32, device="cuda")  # 256-byte aligned
    cmb.check("cmb_fill_uniform_f32", dptr(base), n + 8, ctypes.c_uint64(303), stream_handle(cuda))
    x = base[offset:offset + n]
    assert x.data_ptr() % 32 == 4 * offset
    _check_equal(_sum_noalloc(cuda, cmb, x, n), _sum_with_workspace(cuda, cmb, x, n), n)


def test_noalloc_sum_each_device(cuda, cmb):
    """One call per GPU, each with its own device current: every device has
    its own copy of the scratch array."""
    for d in range(min(cuda.cuda.device_count(), 8)):
        with cuda.cuda.device(d):
            n = (1 << 21) + d
            x = cuda.empty(n, dtype=cuda.float32, device=f"cuda:{d}")
            cmb.check("cmb_fill_uniform_f32", dptr(x), n, ctypes.c_uint64(404 + d),
                      stream_handle(cuda))
            _check_equal(_sum_noalloc(cuda, cmb, x, n), _sum_with_workspace(cuda, cmb, x, n), n)


def test_noalloc_sum_rejects_null_output(cuda, cmb):
    x = cuda.zeros(16, dtype=cuda.float32, device="cuda")
    assert cmb.lib.cmb_stream_sum_f32_noalloc(dptr(x), 16, None, stream_handle(cuda)) == 1


# Runs in a child process that touches the GPU only through the library (and
# the driver API for reading results back), so the reset does not pull the
# device out from under this process's torch context.
_RESET_CHILD = r"""
import ctypes, json, sys
lib = ctypes.CDLL(sys.argv[1])
cu = ctypes.CDLL("libcuda.so.1")
P, SZ = ctypes.c_void_p, ctypes.c_size_t
lib.cmb_last_error.restype = ctypes.c_char_p
lib.cmb_stream_sum_workspace_bytes.restype = SZ
lib.cmb_stream_sum_workspace_bytes.argtypes = [SZ]
lib.cmb_p2p_alloc.argtypes = [SZ, P]
lib.cmb_p2p_free.argtypes = [P]
lib.cmb_fill_uniform_f32.argtypes = [P, SZ, ctypes.c_uint64, P]
lib.cmb_stream_sum_f32.argtypes = [P, SZ, P, P, SZ, P]
lib.cmb_stream_sum_f32_noalloc.argtypes = [P, SZ, P, P]
cu.cuMemcpyDtoH_v2.argtypes = [P, ctypes.c_uint64, SZ]

def check(rc, what):
    if rc != 0:
        raise SystemExit(f"{what}: status {rc}: {lib.cmb_last_error().decode()}")

def alloc(nbytes):
    p = P()
    check(lib.cmb_p2p_alloc(nbytes, ctypes.byref(p)), "cmb_p2p_alloc")
    return p

def read_f64(addr):
    check(cu.cuCtxSynchronize(), "cuCtxSynchronize")
    v = ctypes.c_double()
    check(cu.cuMemcpyDtoH_v2(ctypes.byref(v), addr, 8), "cuMemcpyDtoH")
    return v.value

def both_sums(n, seed):
    x = alloc(4 * n)
    ws_bytes = lib.cmb_stream_sum_workspace_bytes(n)
    ws = alloc(ws_bytes)
    out = alloc(16)
    check(lib.cmb_fill_uniform_f32(x, n, seed, None), "fill")
    check(lib.cmb_stream_sum_f32(x, n, out, ws, ws_bytes, None), "sum")
    ref = read_f64(out.value)
    check(lib.cmb_stream_sum_f32_noalloc(x, n, P(out.value + 8), None), "noalloc sum")
    got = read_f64(out.value + 8)
    for p in (x, ws, out):
        check(lib.cmb_p2p_free(p), "cmb_p2p_free")
    return [ref, got]

n, seed = (1 << 24) + 7, 505
first = both_sums(n, seed)
check(lib.cmb_device_reset(), "cmb_device_reset")
second = both_sums(n, seed)
print(json.dumps({"before_reset": first, "after_reset": second}))
"""


def test_noalloc_sum_after_device_reset(cmb):
    """Call, reset the device through the library, call again: the second
    noalloc call must find the reloaded scratch array."""
    r = subprocess.run([sys.executable, "-c", _RESET_CHILD, cmb.library_path],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    res = json.loads(r.stdout.strip().splitlines()[-1])
    ref, got = res["before_reset"]
    ref2, got2 = res["after_reset"]
    _check_equal(got, ref, "before reset")
    _check_equal(got2, ref2, "after reset")
    assert ref2 == ref
