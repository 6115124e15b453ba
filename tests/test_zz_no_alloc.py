"""GPU test of cmb_stream_sum_f32_noalloc, the read-stream sum for callers
that cannot allocate device memory (their device memory is owned by another
allocator, or they cannot afford cudaMalloc/cudaFree on the path).  It must
give the same sum as cmb_stream_sum_f32, which uses a caller-allocated
workspace, on two calls in a row: the second call reuses the library's
static scratch left over from the first.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.  It passes alone in a fresh
process and after the other tests."""

import ctypes

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


def test_noalloc_sum_matches_workspace_sum_twice(cuda, cmb):
    assert cmb.lib.cmb_stream_sum_noalloc_max_ctas() == 4096
    cases = [((1 << 26) + 3, 101), ((1 << 20) + 17, 202)]  # two calls in a row
    for n, seed in cases:
        x = cuda.empty(n, dtype=cuda.float32, device="cuda")
        cmb.check("cmb_fill_uniform_f32", dptr(x), n, ctypes.c_uint64(seed), stream_handle(cuda))
        ref = _sum_with_workspace(cuda, cmb, x, n)
        got = _sum_noalloc(cuda, cmb, x, n)
        assert np.isfinite(got)
        assert abs(got - ref) <= REL_TOL_SUM * abs(ref), (n, got, ref)
        # same kernel and launch shape: the sums agree exactly
        assert got == ref, (n, got, ref)


def test_noalloc_sum_rejects_null_output(cuda, cmb):
    x = cuda.zeros(16, dtype=cuda.float32, device="cuda")
    assert cmb.lib.cmb_stream_sum_f32_noalloc(dptr(x), 16, None, stream_handle(cuda)) == 1
