"""GPU parity of the HBM streams (reference src/mem_global.cu): copies are
bit-exact, sums match the oracle's fp64 sum within rel 1e-5."""

import ctypes

import numpy as np
import pytest

from oracle import ptr
from tests.helpers import dptr, hptr, stream_handle

pytestmark = pytest.mark.gpu

REL_TOL_SUM = 1e-5  # stated tolerance of the read/sum stream


def test_fill_uniform_matches_oracle(cuda, cmb, orc):
    n = (1 << 20) + 3
    d = cuda.empty(n, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_fill_uniform_f32", dptr(d), n, ctypes.c_uint64(77), stream_handle(cuda))
    ref = np.empty(n, np.float32)
    orc.orc_fill_uniform_f32(ptr(ref), n, 77)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_fill_hash_and_bytes_match_oracle(cuda, cmb, orc):
    n = 100003
    d = cuda.empty(n, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_fill_hash_u32", dptr(d), n, stream_handle(cuda))
    ref = np.empty(n, np.uint32)
    orc.orc_fill_hash_u32(ptr(ref), n)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), ref)
    for off, nb in [(0, 4099), (3, 1000)]:
        b = cuda.zeros(nb + 8, dtype=cuda.uint8, device="cuda")
        cmb.check("cmb_fill_bytes", ctypes.c_void_p(b.data_ptr() + off), nb, ctypes.c_uint64(5),
                  stream_handle(cuda))
        rb = np.empty(nb, np.uint8)
        orc.orc_fill_bytes(ptr(rb), nb, 5)
        assert np.array_equal(b.cpu().numpy()[off:off + nb], rb)


@pytest.mark.parametrize("nbytes", [0, 1, 15, 16, 17, 31, 32, 4096 + 5, (1 << 22) + 48, 3 << 20])
@pytest.mark.parametrize("offset", [0, 16, 4])
def test_copy_bit_exact(cuda, cmb, nbytes, offset):
    src = cuda.randint(0, 256, (nbytes + 64,), dtype=cuda.uint8, device="cuda")
    dst = cuda.zeros(nbytes + 64, dtype=cuda.uint8, device="cuda")
    cmb.check("cmb_stream_copy", ctypes.c_void_p(dst.data_ptr() + offset),
              ctypes.c_void_p(src.data_ptr() + offset), nbytes, stream_handle(cuda))
    cuda.cuda.synchronize()
    assert cuda.equal(dst[offset:offset + nbytes], src[offset:offset + nbytes])
    # nothing outside the range is touched
    assert int(dst[:offset].count_nonzero()) == 0
    assert int(dst[offset + nbytes:].count_nonzero()) == 0


@pytest.mark.parametrize("vec,unroll,ctas", [(16, 1, 8), (16, 8, 2), (32, 2, 4), (32, 8, 1)])
def test_copy_tuned_shapes_bit_exact(cuda, cmb, vec, unroll, ctas):
    n = (7 << 20) + 96
    src = cuda.randint(0, 256, (n,), dtype=cuda.uint8, device="cuda")
    dst = cuda.zeros(n, dtype=cuda.uint8, device="cuda")
    cmb.check("cmb_stream_copy_tuned", dptr(dst), dptr(src), n, vec, unroll, ctas,
              stream_handle(cuda))
    cuda.cuda.synchronize()
    assert cuda.equal(dst, src)


def test_copy_rejects_bad_shape(cuda, cmb):
    a = cuda.empty(64, dtype=cuda.uint8, device="cuda")
    assert cmb.lib.cmb_stream_copy_tuned(dptr(a), dptr(a), 64, 8, 1, 1, stream_handle(cuda)) == 1
    assert cmb.lib.cmb_stream_copy(None, dptr(a), 64, stream_handle(cuda)) == 1


def test_copy_full_size_1gib(cuda, cmb):
    """Config: fp32[2^28] uniform [-1,1) copied to a second buffer, bit-exact."""
    n = 1 << 28
    src = cuda.empty(n, dtype=cuda.float32, device="cuda")
    dst = cuda.empty(n, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_fill_uniform_f32", dptr(src), n, ctypes.c_uint64(2024), stream_handle(cuda))
    dst.fill_(7.0)
    cmb.check("cmb_stream_copy", dptr(dst), dptr(src), 4 * n, stream_handle(cuda))
    cuda.cuda.synchronize()
    assert cuda.equal(src.view(cuda.int32), dst.view(cuda.int32))


def test_copy_headline_size_and_past_4gib(cuda, cmb):
    """The bench's per-GPU workload (fp32[2^30], 4 GiB) and a copy whose
    byte count passes 2^32 with a ragged tail: 64-bit offsets throughout."""
    nbytes = (1 << 32) + 4096 + 36
    src = cuda.empty(nbytes // 4 + 1, dtype=cuda.float32, device="cuda")
    dst = cuda.zeros(nbytes // 4 + 2, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_fill_uniform_f32", dptr(src), src.numel(), ctypes.c_uint64(77),
              stream_handle(cuda))
    for n in (1 << 32, nbytes):
        cmb.check("cmb_stream_copy", dptr(dst), dptr(src), n, stream_handle(cuda))
        cuda.cuda.synchronize()
        a, b = src.view(cuda.uint8)[:n], dst.view(cuda.uint8)[:n]
        assert cuda.equal(a, b)
    assert int(dst.view(cuda.uint8)[nbytes:].count_nonzero()) == 0


def _sum(cuda, cmb, t, n=None, offset_elems=0):
    n = t.numel() - offset_elems if n is None else n
    ws_bytes = cmb.lib.cmb_stream_sum_workspace_bytes(n)
    ws = cuda.empty(ws_bytes, dtype=cuda.uint8, device="cuda")
    out = cuda.full((1,), float("nan"), dtype=cuda.float64, device="cuda")
    cmb.check("cmb_stream_sum_f32", ctypes.c_void_p(t.data_ptr() + 4 * offset_elems), n, dptr(out),
              dptr(ws), ws_bytes, stream_handle(cuda))
    return float(out.item())


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 1000, 65536 + 13, (1 << 22) + 5])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_sum_matches_oracle(cuda, cmb, orc, n, offset):
    total = n + offset
    host = np.empty(max(total, 1), np.float32)
    orc.orc_fill_uniform_f32(ptr(host), host.size, 11)
    d = cuda.from_numpy(host).cuda()
    got = _sum(cuda, cmb, d, n=n, offset_elems=offset)
    part = host[offset:offset + n].copy()  # named: ptr() does not keep the array alive
    ref = orc.orc_sum_f64(ptr(part), n, 0) if n else 0.0
    assert abs(got - ref) <= REL_TOL_SUM * max(abs(ref), 1e-30) or abs(got - ref) < 1e-9


def test_sum_full_size_and_deterministic(cuda, cmb, orc):
    """Config: sum of fp32[2^28] uniform [-1,1) vs the oracle's fp64 sum."""
    n = 1 << 28
    d = cuda.empty(n, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_fill_uniform_f32", dptr(d), n, ctypes.c_uint64(2024), stream_handle(cuda))
    a = _sum(cuda, cmb, d)
    b = _sum(cuda, cmb, d)
    assert a == b  # fixed combine order
    host = d.cpu().numpy()
    ref = orc.orc_sum_f64(ptr(host), n, 0)
    assert abs(ref) > 100.0  # the seed gives a sum well away from 0
    assert abs(a - ref) <= REL_TOL_SUM * abs(ref), (a, ref)
    # linearity: sum(x) computed on halves adds up
    h = n // 2
    s1 = _sum(cuda, cmb, d, n=h)
    s2 = _sum(cuda, cmb, d, n=n - h, offset_elems=h)
    assert abs((s1 + s2) - ref) <= REL_TOL_SUM * abs(ref)


def test_sum_past_4gib(cuda, cmb, orc):
    """fp32[2^30 + 5]: the element count's byte size passes 2^32."""
    n = (1 << 30) + 5
    d = cuda.empty(n, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_fill_uniform_f32", dptr(d), n, ctypes.c_uint64(99), stream_handle(cuda))
    got = _sum(cuda, cmb, d)
    host = d.cpu().numpy()
    ref = orc.orc_sum_f64(ptr(host), n, 0)
    assert abs(got - ref) <= REL_TOL_SUM * max(abs(ref), 1.0), (got, ref)


@pytest.mark.parametrize("n", [1000, (1 << 22) + 3, 1 << 28])
def test_sum_reads_only_this_calls_partials(cuda, cmb, orc, n):
    """A workspace full of NaN bytes before one call: the combine must read
    only the partials this call's sum grid wrote (it waits for that grid)."""
    d = cuda.empty(n, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_fill_uniform_f32", dptr(d), n, ctypes.c_uint64(n), stream_handle(cuda))
    ws_bytes = cmb.lib.cmb_stream_sum_workspace_bytes(n)
    ws = cuda.full((ws_bytes,), 0xFF, dtype=cuda.uint8, device="cuda")
    out = cuda.full((1,), float("nan"), dtype=cuda.float64, device="cuda")
    cmb.check("cmb_stream_sum_f32", dptr(d), n, dptr(out), dptr(ws), ws_bytes, stream_handle(cuda))
    got = float(out.item())
    host = d.cpu().numpy()
    ref = orc.orc_sum_f64(ptr(host), n, 0)
    assert abs(got - ref) <= REL_TOL_SUM * max(abs(ref), 1.0), (got, ref)


def test_sum_rejects_small_workspace(cuda, cmb):
    d = cuda.zeros(1024, dtype=cuda.float32, device="cuda")
    ws = cuda.empty(16, dtype=cuda.uint8, device="cuda")
    out = cuda.empty(1, dtype=cuda.float64, device="cuda")
    rc = cmb.lib.cmb_stream_sum_f32(dptr(d), 1024, dptr(out), dptr(ws), 16, stream_handle(cuda))
    assert rc == 1 and b"workspace" in cmb.lib.cmb_last_error()


def test_copy_host_buffers(cuda, cmb):
    n = (40 << 20) + 16
    src = np.random.default_rng(3).integers(0, 256, n, dtype=np.uint8)
    dst = np.zeros(n, np.uint8)
    chunk = 8 << 20
    a = cuda.empty(3 * chunk, dtype=cuda.uint8, device="cuda")
    b = cuda.empty(3 * chunk, dtype=cuda.uint8, device="cuda")
    cmb.check("cmb_stream_copy_host", hptr(dst), hptr(src), n, dptr(a), dptr(b), 3 * chunk, chunk)
    assert np.array_equal(src, dst)


@pytest.mark.parametrize("nbytes,passes,ctas", [(16, 1, 1), (8 << 20, 4, 0), ((1 << 20) + 48, 3, 7),
                                                (48, 1000, 2), (64 << 10, 37, 0)])
def test_l2_read_exact_sum(cuda, cmb, orc, nbytes, passes, ctas):
    words = nbytes // 4
    d = cuda.empty(words, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_fill_hash_u32", dptr(d), words, stream_handle(cuda))
    out = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    cmb.check("cmb_l2_read", dptr(d), nbytes, passes, ctas, dptr(out), stream_handle(cuda))
    ref = np.empty(words, np.uint32)
    orc.orc_fill_hash_u32(ptr(ref), words)
    expect = (int(ref.astype(np.uint64).sum()) * passes) % (1 << 64)
    assert int(out.cpu().numpy().view(np.uint64)[0]) == expect


@pytest.mark.parametrize("nbytes,passes", [(8192, 1), (8192 * 37, 3), (8 << 20, 16),
                                           (64 << 20, 2)])
def test_l2_read_bulk_exact_sum(cuda, cmb, orc, nbytes, passes):
    """The bulk-copy L2 read: every 8 KiB chunk read `passes` times through
    the shared-memory rings (fewer 8 KiB chunks than warps, a ragged share
    per warp, and more than fit in L2), exact word sum against the oracle."""
    words = nbytes // 4
    d = cuda.empty(words, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_fill_hash_u32", dptr(d), words, stream_handle(cuda))
    out = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_l2_read_bulk", dptr(d), nbytes, passes, dptr(out), dptr(status),
              stream_handle(cuda))
    ref = np.empty(words, np.uint32)
    orc.orc_fill_hash_u32(ptr(ref), words)
    expect = (int(ref.astype(np.uint64).sum()) * passes) % (1 << 64)
    assert int(status.item()) == 0
    assert int(out.cpu().numpy().view(np.uint64)[0]) == expect


def test_l2_read_bulk_rejects_ragged_sizes(cuda, cmb):
    d = cuda.zeros(1 << 16, dtype=cuda.int32, device="cuda")
    out = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    s = stream_handle(cuda)
    assert cmb.lib.cmb_l2_read_bulk(dptr(d), 8192 + 16, 1, dptr(out), None, s) == 1
    assert cmb.lib.cmb_l2_read_bulk(dptr(d), 0, 1, dptr(out), None, s) == 1
    assert cmb.lib.cmb_l2_read_bulk(dptr(d), 8192, 0, dptr(out), None, s) == 1
