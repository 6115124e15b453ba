"""GPU parity of the TMA tile probes (reference src/tma.cu): the tile copy
is bit-exact, the load-only pipeline's per-CTA XOR matches the host, and
no wait times out."""

import ctypes

import numpy as np
import pytest

from oracle import ptr
from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu


def _copy(cuda, cmb, src, rows, cols, box=(128, 128), stages=4, ctas=1, guard=256, flags=None):
    dst = cuda.zeros(rows * cols + guard, dtype=cuda.int16, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if flags is None:
        cmb.check("cmb_tma_tile_copy_bf16", dptr(dst), dptr(src), rows, cols, box[0], box[1],
                  stages, ctas, dptr(status), stream_handle(cuda))
    else:
        cmb.check("cmb_tma_tile_copy_tuned", dptr(dst), dptr(src), rows, cols, box[0], box[1],
                  stages, ctas, flags, dptr(status), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    return dst


@pytest.mark.parametrize("rows,cols,box,stages,ctas", [
    (256, 256, (128, 128), 4, 1),
    (200, 136, (128, 128), 4, 1),      # ragged: partial tiles on both edges
    (1000, 1024, (64, 256), 2, 2),
    (777, 520, (32, 128), 8, 1),
    (4096, 4096, (128, 128), 6, 1),
    (3, 8, (128, 128), 3, 1),
])
def test_tile_copy_bit_exact(cuda, cmb, rows, cols, box, stages, ctas):
    src = cuda.randint(-32768, 32767, (rows * cols,), dtype=cuda.int16, device="cuda")
    dst = _copy(cuda, cmb, src, rows, cols, box, stages, ctas)
    assert cuda.equal(dst[: rows * cols], src)
    assert int(dst[rows * cols:].count_nonzero()) == 0  # nothing past the matrix


@pytest.mark.parametrize("flags", [1, 2, 4, 5])
@pytest.mark.parametrize("rows,cols,box,stages,ctas", [
    (256, 256, (128, 128), 4, 1),
    (200, 136, (128, 128), 4, 2),      # ragged: partial tiles on both edges
    (1000, 1024, (64, 256), 2, 2),
    (777, 520, (32, 128), 8, 1),
    (3, 8, (128, 128), 3, 1),
    (4099, 4104, (256, 64), 3, 2),
])
def test_tile_copy_options_bit_exact(cuda, cmb, rows, cols, box, stages, ctas, flags):
    """Contiguous tile runs (bit 0), evict-first (bit 1), load/store-unit
    stores (bit 2), and bits 0 + 2 together."""
    src = cuda.randint(-32768, 32767, (rows * cols,), dtype=cuda.int16, device="cuda")
    dst = _copy(cuda, cmb, src, rows, cols, box, stages, ctas, flags=flags)
    assert cuda.equal(dst[: rows * cols], src)
    assert int(dst[rows * cols:].count_nonzero()) == 0


def test_tile_copy_full_size(cuda, cmb):
    """Config: 16384 x 16384 bf16 N(0,1), 128x128 boxes, 4-stage ring."""
    n = 16384
    src = cuda.empty(n * n, dtype=cuda.int16, device="cuda")
    cmb.check("cmb_fill_normal_bf16", dptr(src), n * n, ctypes.c_uint64(42), ctypes.c_float(1.0),
              stream_handle(cuda))
    dst = _copy(cuda, cmb, src, n, n, guard=0)
    assert cuda.equal(dst, src)
    vals = src[:1 << 20].view(cuda.bfloat16).float()
    assert abs(float(vals.mean())) < 0.01 and abs(float(vals.std()) - 1.0) < 0.01


def test_tile_load_xor(cuda, cmb):
    rows, cols, box = 1024, 768, (128, 128)
    src = cuda.randint(-32768, 32767, (rows * cols,), dtype=cuda.int16, device="cuda")
    words = 4096
    xor = cuda.zeros(words, dtype=cuda.int32, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_tma_tile_load_bf16", dptr(src), rows, cols, box[0], box[1], 4, dptr(xor), words,
              dptr(status), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    got = xor.cpu().numpy().view(np.uint32)
    m = src.cpu().numpy().reshape(rows, cols)
    tiles_x, tiles_y = cols // box[1], rows // box[0]
    tiles = tiles_x * tiles_y
    grid = min(cuda.cuda.get_device_properties(0).multi_processor_count, words, tiles)
    expect = np.zeros(words, np.uint32)
    for t in range(tiles):
        ty, tx = divmod(t, tiles_x)
        first = m[ty * box[0], tx * box[1]: tx * box[1] + 8].copy().view(np.uint32)
        expect[t % grid] ^= np.bitwise_xor.reduce(first)
    assert np.array_equal(got, expect)


@pytest.mark.parametrize("offset", [0, 16, 1008])
def test_tma_1d_latency(cuda, cmb, orc, offset):
    """The reference's 16-byte 1-D TMA round trip (src/tma.cu:20-69), 256
    times into one zeroed shared-memory slot: the bytes left there must be
    the source's bytes at the load's coordinate (seeded bytes, oracle)."""
    buf = cuda.empty(1024, dtype=cuda.uint8, device="cuda")
    cmb.check("cmb_fill_bytes", dptr(buf), 1024, ctypes.c_uint64(77), stream_handle(cuda))
    cyc = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    landed = cuda.zeros(16, dtype=cuda.uint8, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_tma_1d_latency", dptr(buf), 1024, offset, 256, dptr(cyc), dptr(landed),
              dptr(status), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    ref = np.empty(1024, np.uint8)
    orc.orc_fill_bytes(ptr(ref), 1024, 77)
    assert np.array_equal(landed.cpu().numpy(), ref[offset:offset + 16])
    per = int(cyc.item()) / 256
    assert 50 < per < 20000, per


def test_tma_1d_latency_rejects_unaligned_offset(cuda, cmb):
    buf = cuda.zeros(1024, dtype=cuda.uint8, device="cuda")
    cyc = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    s = stream_handle(cuda)
    for off in (8, 1016, 1024):  # not a multiple of 16, or past the end
        assert cmb.lib.cmb_tma_1d_latency(dptr(buf), 1024, off, 4, dptr(cyc), None, None, s) == 1


@pytest.mark.parametrize("rows,cols,box,stages", [
    (64, 100, (64, 64), 4),     # cols not a multiple of 8
    (64, 64, (64, 64), 9),      # too many stages
    (64, 64, (300, 64), 2),     # box too tall
    (64, 64, (8, 8), 2),        # box bytes not a multiple of 1024
])
def test_tile_copy_rejects_bad_shapes(cuda, cmb, rows, cols, box, stages):
    a = cuda.zeros(rows * cols, dtype=cuda.int16, device="cuda")
    rc = cmb.lib.cmb_tma_tile_copy_bf16(dptr(a), dptr(a), rows, cols, box[0], box[1], stages, 1,
                                        None, stream_handle(cuda))
    assert rc == 1
