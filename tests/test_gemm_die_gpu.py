"""GPU tests of the die map and the GEMMs' die-split tile order.

cmb_sm_die_map must split the SMs cleanly in two (a B200 is two dies), the
same way on a second call.  With a map installed, every GEMM variant must
give C bit-identical to the plain persistent order: the map only decides
which cluster computes which tile, never how a tile is computed.  That must
hold for the measured map and for maps that are wrong on purpose, across
many launches in a row (the claim counters reset themselves), on two
streams at once, and when a captured launch is replayed."""

import ctypes

import numpy as np
import pytest

from tests.helpers import dptr, stream_handle
from tests.test_gemm_gpu import _check_tiles, _normal_bf16, config_tiles

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def die_map(cuda, cmb):
    labels, near, far = cmb.sm_die_map(stream_handle(cuda))
    yield labels, near, far
    cmb.set_sm_die_map(None)


@pytest.fixture
def no_map_after(cmb):
    yield
    cmb.set_sm_die_map(None)


def _operands(cuda, cmb, M, N, K, fp8, seed):
    A = _normal_bf16(cuda, cmb, M, K, seed, 1.0)
    B = _normal_bf16(cuda, cmb, N, K, seed + 1, 1.0)
    if not fp8:
        return A, B, None
    qa = cuda.empty(M * K, dtype=cuda.uint8, device="cuda")
    qb = cuda.empty(N * K, dtype=cuda.uint8, device="cuda")
    sa = cuda.zeros(2, dtype=cuda.float32, device="cuda")
    sb = cuda.zeros(2, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_quantize_e4m3", dptr(A), M * K, dptr(qa), dptr(sa), stream_handle(cuda))
    cmb.check("cmb_quantize_e4m3", dptr(B), N * K, dptr(qb), dptr(sb), stream_handle(cuda))
    return qa, qb, (sa, sb)


def _run(cuda, cmb, ops, M, N, K, fp8, cg, C=None, bf16_out=False, tile_n=0, stream=None):
    A, B, sc = ops
    if C is None:
        C = cuda.full((M * N,), float("nan"), dtype=cuda.bfloat16 if bf16_out else cuda.float32,
                      device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    s = stream if stream is not None else stream_handle(cuda)
    sa = dptr(sc[0]) if fp8 else None
    sb = dptr(sc[1]) if fp8 else None
    if bf16_out:
        cmb.check("cmb_gemm_bf16_out", dptr(A), dptr(B), dptr(C), M, N, K, fp8, sa, sb,
                  dptr(status), s)
    else:
        cmb.check("cmb_gemm_tuned", dptr(A), dptr(B), dptr(C), M, N, K, fp8, sa, sb, cg, 0, 0, 0,
                  tile_n, 0, dptr(status), s)
    return C, status


def _plain_and_split(cuda, cmb, labels, ops, M, N, K, fp8, cg, **kw):
    cmb.set_sm_die_map(None)
    ref, st0 = _run(cuda, cmb, ops, M, N, K, fp8, cg, **kw)
    cmb.set_sm_die_map(labels)
    got, st1 = _run(cuda, cmb, ops, M, N, K, fp8, cg, **kw)
    cuda.cuda.synchronize()
    assert int(st0.item()) == 0 and int(st1.item()) == 0
    return ref, got


def test_die_map_splits_the_sms_in_two(cuda, cmb, die_map):
    labels, near, far = die_map
    sms = cuda.cuda.get_device_properties(0).multi_processor_count
    present = labels[labels != 0xFF]
    assert set(np.unique(present)) == {0, 1}
    assert len(present) == sms
    n0, n1 = int((present == 0).sum()), int((present == 1).sum())
    assert min(n0, n1) >= sms // 3, (n0, n1)  # two dies of similar size
    assert labels[np.flatnonzero(labels != 0xFF)[0]] == 0  # die 0 holds the lowest id
    assert 100 < far - near < 2000 and 200 < near < 2000, (near, far)
    again, _, _ = cmb.sm_die_map(stream_handle(cuda))
    assert np.array_equal(again, labels)


@pytest.mark.parametrize("fp8", [0, 1])
@pytest.mark.parametrize("cg,tile_n", [(2, 0), (1, 0), (2, 256)])
def test_die_split_8192_is_bit_identical(cuda, cmb, orc, die_map, no_map_after, fp8, cg, tile_n):
    M = N = K = 8192
    ops = _operands(cuda, cmb, M, N, K, fp8, 71)
    ref, got = _plain_and_split(cuda, cmb, die_map[0], ops, M, N, K, fp8, cg, tile_n=tile_n)
    assert cuda.equal(ref, got)
    if fp8 == 0 and cg == 2 and tile_n == 0:  # and the split result against the oracle
        A_h = ops[0].cpu().numpy().view(np.uint16)
        B_h = ops[1].cpu().numpy().view(np.uint16)
        C = got.cpu().numpy().reshape(M, N)
        _check_tiles(orc, A_h, B_h, C, K, config_tiles(M, N, 72, count=16))


@pytest.mark.parametrize("fp8", [0, 1])
def test_die_split_bf16_out_is_bit_identical(cuda, cmb, die_map, no_map_after, fp8):
    M, N, K = 8192, 8192, 4096
    ops = _operands(cuda, cmb, M, N, K, fp8, 73)
    ref, got = _plain_and_split(cuda, cmb, die_map[0], ops, M, N, K, fp8, 2, bf16_out=True)
    assert cuda.equal(ref, got)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(1000, 700, 512), (6144, 8192, 1024), (256, 512, 64),
                                   (4096, 4600, 208)])
def test_die_split_ragged_and_few_tiles(cuda, cmb, die_map, no_map_after, cg, M, N, K):
    ops = _operands(cuda, cmb, M, N, K, 0, 74)
    ref, got = _plain_and_split(cuda, cmb, die_map[0], ops, M, N, K, 0, cg)
    assert cuda.equal(ref, got)


def _wrong_maps(labels, seed):
    ids = np.flatnonzero(labels != 0xFF)
    maps = {}
    m = labels.copy(); m[ids] = 1 - labels[ids]; maps["inverted"] = m
    m = labels.copy(); m[ids] = ids % 2; maps["id_parity"] = m
    m = labels.copy(); m[ids] = 0; m[ids[:2]] = 1; maps["two_sms_on_die_1"] = m
    m = labels.copy(); m[ids] = np.random.default_rng(seed).integers(0, 2, len(ids)); maps["random"] = m
    return maps


@pytest.mark.parametrize("cg", [1, 2])
def test_die_split_with_wrong_maps(cuda, cmb, die_map, no_map_after, cg):
    """The map is a placement hint: a map that does not match the hardware
    moves tiles between clusters but computes every tile once."""
    M, N, K = 4096, 4096, 1024
    ops = _operands(cuda, cmb, M, N, K, 0, 75)
    for name, m in _wrong_maps(die_map[0], 76).items():
        ref, got = _plain_and_split(cuda, cmb, m, ops, M, N, K, 0, cg)
        assert cuda.equal(ref, got), name


def test_die_split_many_launches_and_two_streams(cuda, cmb, die_map, no_map_after):
    """More launches than there are claim slots (each slot's counters must
    be back at zero when it comes round again), on two streams at once."""
    M, N, K = 2048, 2048, 512
    ops = _operands(cuda, cmb, M, N, K, 0, 77)
    cmb.set_sm_die_map(None)
    ref, _ = _run(cuda, cmb, ops, M, N, K, 0, 2)
    cmb.set_sm_die_map(die_map[0])
    streams = [cuda.cuda.Stream(), cuda.cuda.Stream()]
    outs = [cuda.empty(M * N, dtype=cuda.float32, device="cuda") for _ in range(4)]
    statuses = []
    cuda.cuda.synchronize()
    for i in range(150):
        s = streams[i % 2]
        C = outs[i % 4]
        with cuda.cuda.stream(s):
            _, st = _run(cuda, cmb, ops, M, N, K, 0, 2, C=C, stream=ctypes.c_void_p(s.cuda_stream))
        statuses.append(st)
        if i % 4 == 3:
            cuda.cuda.synchronize()
            assert all(int(st.item()) == 0 for st in statuses)
            statuses.clear()
            for C in outs:
                assert cuda.equal(C, ref)
                C.fill_(float("nan"))
            cuda.cuda.synchronize()  # the fills finish before the next launches
    cuda.cuda.synchronize()


def test_die_split_graph_replay(cuda, cmb, die_map, no_map_after):
    """A captured launch keeps its claim slot; its counters are back at zero
    after every replay, so each replay computes every tile."""
    M, N, K = 4096, 4096, 512
    ops = _operands(cuda, cmb, M, N, K, 0, 78)
    cmb.set_sm_die_map(None)
    ref, _ = _run(cuda, cmb, ops, M, N, K, 0, 2)
    cmb.set_sm_die_map(die_map[0])
    C = cuda.empty(M * N, dtype=cuda.float32, device="cuda")
    _run(cuda, cmb, ops, M, N, K, 0, 2, C=C)  # sets the kernel attributes before capture
    cuda.cuda.synchronize()
    g = cuda.cuda.CUDAGraph()
    with cuda.cuda.graph(g, capture_error_mode="relaxed"):
        _, st = _run(cuda, cmb, ops, M, N, K, 0, 2, C=C)
    for _ in range(3):
        C.fill_(float("nan"))
        g.replay()
        cuda.cuda.synchronize()
        assert int(st.item()) == 0
        assert cuda.equal(C, ref)
    del g
