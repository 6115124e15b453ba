"""GPU parity of the tcgen05 GEMM probes against the oracle's fp64 GEMM
(stated tolerance: per checked tile, max |C - C_ref| <= 1e-2 * max |C_ref|,
the max-norm reading of "rel tol 1e-2"), and of the e4m3 quantiser against
the oracle's encoder (bit-exact).  The 8192^3 configuration is checked on 64
sampled 256 x 256 output tiles (the two corner tiles included) of every
variant the bench reports: bf16 and e4m3, fp32 and bf16 C, 1-CTA 128 x 256,
2-CTA 256 x 512 and 2-CTA 256 x 256 tiles."""

import ctypes

import numpy as np
import pytest

from oracle import ptr
from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu

RTOL = 1e-2  # stated GEMM tolerance (max-norm, per tile)


def _normal_bf16(cuda, cmb, rows, cols, seed, scale):
    t = cuda.empty(rows * cols, dtype=cuda.int16, device="cuda")
    cmb.check("cmb_fill_normal_bf16", dptr(t), rows * cols, ctypes.c_uint64(seed),
              ctypes.c_float(scale), stream_handle(cuda))
    return t


def _gemm(cuda, cmb, fn, A, B, M, N, K, cg, scales=None):
    C = cuda.full((M * N,), float("nan"), dtype=cuda.float32, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if fn == "bf16":
        cmb.check("cmb_gemm_bf16", dptr(A), dptr(B), dptr(C), M, N, K, cg, dptr(status),
                  stream_handle(cuda))
    else:
        cmb.check("cmb_gemm_e4m3", dptr(A), dptr(B), dptr(C), M, N, K, dptr(scales[0]),
                  dptr(scales[1]), cg, dptr(status), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0, "a device-side wait timed out"
    return C.cpu().numpy().reshape(M, N)


def _check_tiles(orc, A_h, B_h, C, K, tiles, dtype=0, sa=1.0, sb=1.0):
    """Max over `tiles` of the per-tile max-norm relative error against the
    oracle's fp64 GEMM (all tiles computed at once on the host's threads)."""
    spec = np.array(tiles, np.int32).reshape(-1, 4)
    ref_all = np.empty(int((spec[:, 2].astype(np.int64) * spec[:, 3]).sum()), np.float64)
    orc.orc_gemm_tiles_f64(ptr(A_h), ptr(B_h), dtype, K, K, K, len(spec), ptr(spec), sa, sb,
                           ptr(ref_all), 0)
    worst, off = 0.0, 0
    for (r0, c0, tm, tn) in tiles:
        ref = ref_all[off:off + tm * tn].reshape(tm, tn)
        off += tm * tn
        got = C[r0:r0 + tm, c0:c0 + tn].astype(np.float64)
        assert np.isfinite(got).all()
        err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
        worst = max(worst, err)
        assert err <= RTOL, (r0, c0, err)
    return worst


def config_tiles(M, N, seed, count=64, size=256):
    """`count` sampled size x size output tiles on a size-aligned grid: the
    first and the last corner tile, the rest drawn from `seed`."""
    rng = np.random.default_rng(seed)
    tiles = [(int(r) * size, int(c) * size, size, size)
             for r, c in zip(rng.integers(0, M // size, count), rng.integers(0, N // size, count))]
    tiles[0] = (0, 0, size, size)
    tiles[1] = (M - size, N - size, size, size)
    return tiles


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (256, 512, 1024), (200, 136, 72),
                                   (1000, 700, 520), (128, 256, 8), (96, 130, 64)])
def test_gemm_bf16_small_full_check(cuda, cmb, orc, cg, M, N, K):
    A = _normal_bf16(cuda, cmb, M, K, 1, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 2, K ** -0.5)
    C = _gemm(cuda, cmb, "bf16", A, B, M, N, K, cg)
    A_h = A.cpu().numpy().view(np.uint16)
    B_h = B.cpu().numpy().view(np.uint16)
    worst = _check_tiles(orc, A_h, B_h, C, K, [(0, 0, M, N)])
    assert worst < 1e-4  # fp32 accumulation of exact bf16 products


@pytest.mark.parametrize("cg", [1, 2])
def test_gemm_bf16_8192_sampled_tiles(cuda, cmb, orc, cg):
    """Config: M=N=K=8192, A/B bf16 N(0,1)*K^-0.5; 64 sampled 256x256 output
    tiles against the fp64 oracle."""
    M = N = K = 8192
    A = _normal_bf16(cuda, cmb, M, K, 11, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 12, K ** -0.5)
    C = _gemm(cuda, cmb, "bf16", A, B, M, N, K, cg)
    A_h = A.cpu().numpy().view(np.uint16)
    B_h = B.cpu().numpy().view(np.uint16)
    worst = _check_tiles(orc, A_h, B_h, C, K, config_tiles(M, N, cg))
    assert worst < 1e-4
    assert np.isfinite(C).all()


def _quantize(cuda, cmb, x):
    q = cuda.empty(x.numel(), dtype=cuda.uint8, device="cuda")
    sc = cuda.zeros(2, dtype=cuda.float32, device="cuda")
    cmb.check("cmb_quantize_e4m3", dptr(x), x.numel(), dptr(q), dptr(sc), stream_handle(cuda))
    return q, sc


def test_quantize_e4m3_matches_oracle(cuda, cmb, orc):
    n = 1 << 20
    x = _normal_bf16(cuda, cmb, 1, n, 5, 3.0)
    q, sc = _quantize(cuda, cmb, x)
    x_h = x.cpu().numpy().view(np.uint16)
    amax = orc.orc_amax_bf16(ptr(x_h), n)
    s = sc.cpu().numpy()
    assert s[1] == np.float32(amax)
    assert s[0] == np.float32(amax) / np.float32(448.0)
    inv = np.float32(448.0) / np.float32(amax)
    ref = np.empty(n, np.uint8)
    orc.orc_quantize_e4m3(ptr(x_h), n, float(inv), ptr(ref))
    assert np.array_equal(q.cpu().numpy(), ref)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (384, 520, 1040), (8192, 8192, 8192)])
def test_gemm_e4m3(cuda, cmb, orc, cg, M, N, K):
    """Config (largest case): the 8192^3 GEMM with A, B quantised to e4m3 with
    a per-tensor scale; checked against fp64 on the dequantised inputs."""
    A = _normal_bf16(cuda, cmb, M, K, 21, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 22, K ** -0.5)
    qa, sa = _quantize(cuda, cmb, A)
    qb, sb = _quantize(cuda, cmb, B)
    C = _gemm(cuda, cmb, "e4m3", qa, qb, M, N, K, cg, scales=(sa[:1], sb[:1]))
    qa_h, qb_h = qa.cpu().numpy(), qb.cpu().numpy()
    sa_h, sb_h = float(sa[0].item()), float(sb[0].item())
    tiles = [(0, 0, M, N)] if M * N <= 1 << 20 else config_tiles(M, N, 7 + cg)
    _check_tiles(orc, qa_h, qb_h, C, K, tiles, dtype=1, sa=sa_h, sb=sb_h)


@pytest.mark.parametrize("fp8", [0, 1])
def test_gemm_8192_2cta_256x256_tile(cuda, cmb, orc, fp8):
    """Config, with the configuration's literal 2-CTA 256 x 256 x 64 tile
    (the bench's bf16_8192_2cta_256x256 line): two accumulators of 256
    columns, 4 epilogue warps; 64 sampled 256x256 tiles against fp64."""
    M = N = K = 8192
    A = _normal_bf16(cuda, cmb, M, K, 71, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 72, K ** -0.5)
    C = cuda.full((M * N,), float("nan"), dtype=cuda.float32, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if fp8:
        qa, sa = _quantize(cuda, cmb, A)
        qb, sb = _quantize(cuda, cmb, B)
        args = (dptr(qa), dptr(qb), dptr(C), M, N, K, 1, dptr(sa), dptr(sb))
        a_h, b_h = qa.cpu().numpy(), qb.cpu().numpy()
        s_a, s_b = float(sa[0].item()), float(sb[0].item())
    else:
        args = (dptr(A), dptr(B), dptr(C), M, N, K, 0, None, None)
        a_h, b_h = A.cpu().numpy().view(np.uint16), B.cpu().numpy().view(np.uint16)
        s_a = s_b = 1.0
    cmb.check("cmb_gemm_tuned", *args, 2, 4, 8, 2, 256, 4, dptr(status), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    _check_tiles(orc, a_h, b_h, C.cpu().numpy().reshape(M, N), K, config_tiles(M, N, 9 + fp8),
                 dtype=fp8, sa=s_a, sb=s_b)


@pytest.mark.parametrize("fp8", [0, 1])
@pytest.mark.parametrize("cg,stages,epi,tile_n,ew", [
    (1, 3, 1, 256, 4), (1, 4, 2, 256, 4), (2, 4, 1, 256, 4), (2, 5, 2, 256, 4), (2, 6, 2, 256, 4),
    (2, 7, 1, 256, 4), (2, 3, 2, 512, 4), (2, 4, 2, 512, 4), (2, 4, 1, 512, 4), (2, 3, 2, 512, 8),
    (2, 4, 1, 512, 8), (2, 4, 2, 512, 8)])
def test_gemm_tuned_shapes(cuda, cmb, orc, fp8, cg, stages, epi, tile_n, ew):
    M, N, K = 700, 520, 1040
    A = _normal_bf16(cuda, cmb, M, K, 31, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 32, K ** -0.5)
    C = cuda.full((M * N,), float("nan"), dtype=cuda.float32, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if fp8:
        qa, sa = _quantize(cuda, cmb, A)
        qb, sb = _quantize(cuda, cmb, B)
        cmb.check("cmb_gemm_tuned", dptr(qa), dptr(qb), dptr(C), M, N, K, 1, dptr(sa), dptr(sb), cg,
                  stages, 4, epi, tile_n, ew, dptr(status), stream_handle(cuda))
        a_h, b_h, dt = qa.cpu().numpy(), qb.cpu().numpy(), 1
        s_a, s_b = float(sa[0].item()), float(sb[0].item())
    else:
        cmb.check("cmb_gemm_tuned", dptr(A), dptr(B), dptr(C), M, N, K, 0, None, None, cg, stages,
                  4, epi, tile_n, ew, dptr(status), stream_handle(cuda))
        a_h, b_h, dt = A.cpu().numpy().view(np.uint16), B.cpu().numpy().view(np.uint16), 0
        s_a = s_b = 1.0
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    _check_tiles(orc, a_h, b_h, C.cpu().numpy().reshape(M, N), K, [(0, 0, M, N)], dtype=dt,
                 sa=s_a, sb=s_b)


@pytest.mark.parametrize("fp8", [0, 1])
@pytest.mark.parametrize("epi", [1, 2])
@pytest.mark.parametrize("M,N,K", [(4096, 4096, 64), (4096, 4600, 208), (6144, 8192, 1024)])
def test_gemm_held_epilogue_many_tiles(cuda, cmb, orc, fp8, epi, M, N, K):
    """256 x 512 tiles with 8 epilogue warps: each half of the accumulator
    is handed back before it is stored, and the next tile's MMAs start on
    half 0 over the stages already loaded.  Sizes give most clusters two or
    more tiles, K shorter than the ring (one K block) and a ragged last K
    block and column edge."""
    A = _normal_bf16(cuda, cmb, M, K, 51, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 52, K ** -0.5)
    C = cuda.full((M * N,), float("nan"), dtype=cuda.float32, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if fp8:
        qa, sa = _quantize(cuda, cmb, A)
        qb, sb = _quantize(cuda, cmb, B)
        args = (dptr(qa), dptr(qb), dptr(C), M, N, K, 1, dptr(sa), dptr(sb))
        a_h, b_h, dt = qa.cpu().numpy(), qb.cpu().numpy(), 1
        s_a, s_b = float(sa[0].item()), float(sb[0].item())
    else:
        args = (dptr(A), dptr(B), dptr(C), M, N, K, 0, None, None)
        a_h, b_h, dt = A.cpu().numpy().view(np.uint16), B.cpu().numpy().view(np.uint16), 0
        s_a = s_b = 1.0
    cmb.check("cmb_gemm_tuned", *args, 2, 4, 8, epi, 512, 8, dptr(status), stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    out = C.cpu().numpy().reshape(M, N)
    assert not np.isnan(out).any()
    rng = np.random.default_rng(M + N + K)
    tiles = [(int(r) * 64, int(c) * 64, 64, 64)
             for r, c in zip(rng.integers(0, M // 64, 48), rng.integers(0, N // 64, 48))]
    tiles.append((M - 64, N - 64, 64, 64))  # the last tile's corner, ragged columns included
    _check_tiles(orc, a_h, b_h, out, K, tiles, dtype=dt, sa=s_a, sb=s_b)


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("epi", [1, 2])
@pytest.mark.parametrize("M,N,K", [(1000, 700, 512), (1024, 700, 64), (1000, 136, 520)])
def test_gemm_ragged_columns(cuda, cmb, orc, cg, epi, M, N, K):
    """Column edges where the last stored box is clipped and the boxes after
    it lie wholly outside C (the staged TMA-store epilogue must not reuse a
    buffer a clipped store is still reading)."""
    A = _normal_bf16(cuda, cmb, M, K, 41, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 42, K ** -0.5)
    C = cuda.full((M * N,), float("nan"), dtype=cuda.float32, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    for _ in range(3):
        cmb.check("cmb_gemm_tuned", dptr(A), dptr(B), dptr(C), M, N, K, 0, None, None, cg, 0, 0, epi,
                  0, 0, dptr(status), stream_handle(cuda))
        cuda.cuda.synchronize()
        assert int(status.item()) == 0
        _check_tiles(orc, A.cpu().numpy().view(np.uint16), B.cpu().numpy().view(np.uint16),
                     C.cpu().numpy().reshape(M, N), K, [(0, 0, M, N)])


@pytest.mark.parametrize("fp8", [0, 1])
def test_mma_rate_constant_operands(cuda, cmb, fp8):
    ctas, iters = 8, 1000
    out = cuda.zeros(ctas * 128, dtype=cuda.float32, device="cuda")
    cyc = cuda.zeros(ctas, dtype=cuda.int64, device="cuda")
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_mma_rate", fp8, iters, ctas, dptr(out), dptr(cyc), dptr(status),
              stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    # ones x ones: each MMA adds K (16 bf16 / 32 e4m3) to every element
    assert bool((out == iters * 4 * (32 if fp8 else 16)).all())
    assert int(cyc.min()) > 0


def test_gemm_rejects_bad_args(cuda, cmb):
    a = cuda.zeros(1024, dtype=cuda.int16, device="cuda")
    c = cuda.zeros(1024, dtype=cuda.float32, device="cuda")
    s = stream_handle(cuda)
    assert cmb.lib.cmb_gemm_bf16(dptr(a), dptr(a), dptr(c), 16, 16, 12, 1, None, s) == 1  # K%8
    assert cmb.lib.cmb_gemm_bf16(dptr(a), dptr(a), dptr(c), 16, 16, 16, 3, None, s) == 1  # cg
    assert cmb.lib.cmb_gemm_bf16(dptr(a), dptr(a), dptr(c), 0, 16, 16, 1, None, s) == 1
    assert cmb.lib.cmb_gemm_e4m3(dptr(a), dptr(a), dptr(c), 16, 16, 16, None, None, 1, None,
                                 s) == 1
    # TMA-store epilogue needs N % 4 == 0; 7 stages only with direct stores
    assert cmb.lib.cmb_gemm_tuned(dptr(a), dptr(a), dptr(c), 16, 18, 16, 0, None, None, 2, 4, 0, 2,
                                  0, 0, None, s) == 1
    assert cmb.lib.cmb_gemm_tuned(dptr(a), dptr(a), dptr(c), 16, 16, 16, 0, None, None, 2, 7, 0, 2,
                                  0, 0, None, s) == 1
    assert cmb.lib.cmb_gemm_tuned(dptr(a), dptr(a), dptr(c), 16, 16, 16, 0, None, None, 1, 4, 0, 2,
                                  512, 0, None, s) == 1


@pytest.mark.parametrize("fp8", [0, 1])
@pytest.mark.parametrize("M,N,K,offset", [
    (256, 512, 256, 0), (700, 520, 1040, 0), (1000, 700, 512, 0), (4096, 4600, 208, 0),
    (512, 1024, 512, 8), (8192, 8192, 8192, 0)])
def test_gemm_bf16_out_is_the_rounded_fp32_result(cuda, cmb, orc, fp8, M, N, K, offset):
    """bf16 C equals the fp32 C of the same GEMM rounded to nearest-even
    bf16, bit for bit (same tiles, same accumulation order), and is within
    the tolerance of the oracle's fp64 product.  N = 700 (N % 8 != 0) and
    an 8-byte-offset C take the direct-store epilogue."""
    A = _normal_bf16(cuda, cmb, M, K, 61, K ** -0.5)
    B = _normal_bf16(cuda, cmb, N, K, 62, K ** -0.5)
    C32 = cuda.full((M * N,), float("nan"), dtype=cuda.float32, device="cuda")
    cb = cuda.full((M * N + 8,), float("nan"), dtype=cuda.bfloat16, device="cuda")
    Cb = cb[offset // 2: offset // 2 + M * N]
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if fp8:
        qa, sa = _quantize(cuda, cmb, A)
        qb, sb = _quantize(cuda, cmb, B)
        ops = (dptr(qa), dptr(qb))
        cmb.check("cmb_gemm_e4m3", *ops, dptr(C32), M, N, K, dptr(sa), dptr(sb), 2, dptr(status),
                  stream_handle(cuda))
        cmb.check("cmb_gemm_bf16_out", *ops, dptr(Cb), M, N, K, 1, dptr(sa), dptr(sb),
                  dptr(status), stream_handle(cuda))
        a_h, b_h, dt = qa.cpu().numpy(), qb.cpu().numpy(), 1
        s_a, s_b = float(sa[0].item()), float(sb[0].item())
    else:
        ops = (dptr(A), dptr(B))
        cmb.check("cmb_gemm_bf16", *ops, dptr(C32), M, N, K, 2, dptr(status), stream_handle(cuda))
        cmb.check("cmb_gemm_bf16_out", *ops, dptr(Cb), M, N, K, 0, None, None, dptr(status),
                  stream_handle(cuda))
        a_h, b_h, dt = A.cpu().numpy().view(np.uint16), B.cpu().numpy().view(np.uint16), 0
        s_a = s_b = 1.0
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    assert cuda.equal(Cb.view(cuda.int16), C32.to(cuda.bfloat16).view(cuda.int16))
    assert cuda.isnan(cb[:offset // 2]).all() and cuda.isnan(cb[offset // 2 + M * N:]).all()
    out = Cb.float().cpu().numpy().reshape(M, N)
    if M * N <= 1 << 20:
        tiles = [(0, 0, M, N)]
    elif M == N == 8192:
        tiles = config_tiles(M, N, 13 + fp8)
    else:
        rng = np.random.default_rng(M + N)
        tiles = [(int(r) * 64, int(c) * 64, 64, 64)
                 for r, c in zip(rng.integers(0, M // 64, 16), rng.integers(0, N // 64, 16))]
    _check_tiles(orc, a_h, b_h, out, K, tiles, dtype=dt, sa=s_a, sb=s_b)
