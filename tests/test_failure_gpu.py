"""Failure detection on the GPU without a fault: a bounded device-side wait
that nothing satisfies returns CMB_ERR_TIMEOUT, and the context stays usable
for the next launch."""

import ctypes

import pytest

from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda, cmb):
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    waited = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    limit = 20_000_000  # 20 ms
    cmb.check("cmb_selftest_wait_timeout", ctypes.c_uint64(limit), dptr(status), dptr(waited),
              stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 3  # CMB_ERR_TIMEOUT
    assert limit <= int(waited.item()) < 50 * limit
    # the context still runs work
    x = cuda.arange(1024, device="cuda", dtype=cuda.float32)
    y = cuda.empty_like(x)
    cmb.check("cmb_stream_copy", dptr(y), dptr(x), 4096, stream_handle(cuda))
    assert cuda.equal(x, y)


def test_selftest_rejects_long_limits(cuda, cmb):
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    waited = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    assert cmb.lib.cmb_selftest_wait_timeout(ctypes.c_uint64(5_000_000_000), dptr(status),
                                             dptr(waited), stream_handle(cuda)) == 1
