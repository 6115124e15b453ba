"""CPU tests of the oracle itself: published test vectors, format round
trips, and the properties the probes rely on (single cycle, exact uniform
grid, fp64 sums)."""

import math

import numpy as np
import pytest

import oracle
from oracle import ptr


def test_splitmix64_published_vector(orc):
    # SplitMix64 seeded with 0: first outputs (Vigna's reference generator).
    assert orc.orc_splitmix64_at(0, 0) == 0xE220A8397B1DCDAF
    assert orc.orc_splitmix64_at(0, 1) == 0x6E789E6AA1B965F4
    assert orc.orc_splitmix64_at(0, 2) == 0x06C45D188009454F


def test_hash32_matches_reference_formula(orc):
    # src/mem_global.cu:7-10 restated in numpy (uint32 wrap-around).
    i = np.arange(0, 1 << 16, dtype=np.uint32)
    with np.errstate(over="ignore"):
        x = i + np.uint32(0x9E3779B9)
        x = (x ^ (x >> np.uint32(16))) * np.uint32(0x85EBCA6B)
        x = (x ^ (x >> np.uint32(13))) * np.uint32(0xC2B2AE35)
        x = x ^ (x >> np.uint32(16))
    out = np.empty_like(i)
    orc.orc_fill_hash_u32(ptr(out), out.size)
    assert np.array_equal(out, x)


def test_uniform_grid_is_exact(orc):
    x = np.empty(1 << 16, np.float32)
    orc.orc_fill_uniform_f32(ptr(x), x.size, 1234)
    assert x.min() >= -1.0 and x.max() < 1.0
    # every value is a multiple of 2^-23
    q = (x.astype(np.float64) + 1.0) * 2.0**23
    assert np.all(q == np.round(q))
    ref = np.array([(orc.orc_splitmix64_at(1234, k) >> 40) * 2.0**-23 - 1.0 for k in range(64)])
    assert np.array_equal(x[:64].astype(np.float64), ref)


def test_bytes_layout(orc):
    b = np.empty(37, np.uint8)
    orc.orc_fill_bytes(ptr(b), b.size, 99)
    words = [orc.orc_splitmix64_at(99, k) for k in range(5)]
    expect = [(words[i // 8] >> (8 * (i % 8))) & 0xFF for i in range(37)]
    assert list(b) == expect


@pytest.mark.parametrize("slots", [1, 2, 3, 64, 4097])
def test_chase_single_cycle(orc, slots):
    links = np.empty(slots * 32, np.uint32)
    orc.orc_chase_build(ptr(links), links.nbytes, 17)
    assert orc.orc_chase_is_single_cycle(ptr(links), links.nbytes) == 1
    # the walk returns to 0 after exactly `slots` hops
    assert orc.orc_chase_walk(ptr(links), slots, 0) == 0
    if slots > 1:
        assert orc.orc_chase_walk(ptr(links), slots - 1, 0) != 0
    heads = links[::32]
    assert np.all(heads % 32 == 0) and np.all(heads < links.size)
    # padding words hold fmix32 of their index (include/memory_chase.h:128-133)
    mask = np.ones(links.size, bool)
    mask[::32] = False
    idx = np.nonzero(mask)[0][:100]
    assert all(links[k] == orc.orc_hash32(int(k)) for k in idx)


def test_chase_detects_broken_cycle(orc):
    links = np.empty(64 * 32, np.uint32)
    orc.orc_chase_build(ptr(links), links.nbytes, 5)
    # plant a short cycle: the first slot links to itself
    links[0] = 0
    assert orc.orc_chase_is_single_cycle(ptr(links), links.nbytes) == 0


def test_sum_f64_matches_fsum(orc):
    x = np.empty(100003, np.float32)
    orc.orc_fill_uniform_f32(ptr(x), x.size, 3)
    for threads in (1, 3, 8):
        s = orc.orc_sum_f64(ptr(x), x.size, threads)
        assert abs(s - math.fsum(x.astype(np.float64))) <= 1e-9 * np.abs(x).sum()


def test_memcpy_mt(orc):
    a = np.arange(1 << 20, dtype=np.uint8)
    b = np.zeros_like(a)
    orc.orc_memcpy_mt(ptr(b), ptr(a), a.size, 4)
    assert np.array_equal(a, b)


def test_bf16_rne(orc):
    vals = np.array([1.0, -2.5, 1.00390625, 1.0078125, 1.01171875, 3.0e38, 1e-40], np.float32)
    for v in vals:
        bits = int(np.float32(v).view(np.uint32))
        lsb = (bits >> 16) & 1
        expect = ((bits + 0x7FFF + lsb) >> 16) & 0xFFFF
        assert orc.orc_f32_to_bf16_rne(float(v)) == expect
    # ties go to even: 1 + 2^-8 is halfway between 1 and 1 + 2^-7
    assert orc.orc_f32_to_bf16_rne(1.00390625) == 0x3F80
    assert orc.orc_f32_to_bf16_rne(1.01171875) == 0x3F82


def test_e4m3_table(orc):
    # OCP E4M3: bias 7, max finite 448, min subnormal 2^-9, 0x7f/0xff NaN.
    assert orc.orc_e4m3_to_f32(0x7E) == 448.0
    assert orc.orc_e4m3_to_f32(0x01) == 2.0**-9
    assert orc.orc_e4m3_to_f32(0x08) == 2.0**-6
    assert orc.orc_e4m3_to_f32(0x38) == 1.0
    assert math.isnan(orc.orc_e4m3_to_f32(0x7F))
    # encode(decode(c)) == c for every finite code
    for c in range(256):
        if c & 0x7F == 0x7F:
            continue
        v = orc.orc_e4m3_to_f32(c)
        got = orc.orc_f32_to_e4m3_satfinite(v)
        assert got == c or (v == 0.0 and got & 0x7F == 0), (c, v, got)


def test_e4m3_rounding(orc):
    # nearest-even between 1.0 (0x38) and 1.125 (0x39): 1.0625 -> 1.0
    assert orc.orc_f32_to_e4m3_satfinite(1.0625) == 0x38
    assert orc.orc_f32_to_e4m3_satfinite(1.0626) == 0x39
    # between 1.125 and 1.25, the tie 1.1875 goes to 1.25 (even mantissa 2)
    assert orc.orc_f32_to_e4m3_satfinite(1.1875) == 0x3A
    # saturation of finite values and of infinity
    assert orc.orc_f32_to_e4m3_satfinite(1000.0) == 0x7E
    assert orc.orc_f32_to_e4m3_satfinite(-1e30) == 0xFE
    assert orc.orc_f32_to_e4m3_satfinite(float("inf")) == 0x7E
    # subnormal rounding: 1.5 * 2^-9 ties to 2 * 2^-9 (even)
    assert orc.orc_f32_to_e4m3_satfinite(1.5 * 2.0**-9) == 0x02
    assert orc.orc_f32_to_e4m3_satfinite(0.4 * 2.0**-9) == 0x00


def test_gemm_tile_f64_matches_numpy(orc):
    rng = np.random.default_rng(0)
    M, N, K = 48, 40, 96
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((N, K)).astype(np.float32)
    a16 = np.array([orc.orc_f32_to_bf16_rne(float(v)) for v in a.ravel()], np.uint16).reshape(M, K)
    b16 = np.array([orc.orc_f32_to_bf16_rne(float(v)) for v in b.ravel()], np.uint16).reshape(N, K)
    af = (a16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    bf = (b16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    out = np.empty((16, 8), np.float64)
    orc.orc_gemm_tile_f64(ptr(a16), ptr(b16), 0, K, K, K, 8, 24, 16, 8, 1.0, 1.0, ptr(out))
    assert np.allclose(out, af[8:24] @ bf[24:32].T, rtol=1e-12, atol=1e-12)
    c = np.empty((M, N), np.float32)
    orc.orc_gemm_bf16_rows_f32(ptr(a16), ptr(b16), ptr(c), N, K, 0, M, 3)
    assert np.allclose(c, af @ bf.T, rtol=1e-4, atol=1e-4)


def test_quantize_e4m3(orc):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(4096).astype(np.float32)
    x16 = np.array([orc.orc_f32_to_bf16_rne(float(v)) for v in x], np.uint16)
    amax = orc.orc_amax_bf16(ptr(x16), x16.size)
    xf = (x16.astype(np.uint32) << 16).view(np.float32)
    assert amax == np.abs(xf).max()
    inv = np.float32(448.0) / np.float32(amax)
    q = np.empty(x16.size, np.uint8)
    orc.orc_quantize_e4m3(ptr(x16), x16.size, float(inv), ptr(q))
    back = np.array([orc.orc_e4m3_to_f32(int(c)) for c in q], np.float32)
    assert np.abs(back).max() <= 448.0
    # relative error of e4m3 normals is at most 2^-4
    big = np.abs(xf * inv) > 2.0**-6
    assert np.all(np.abs(back[big] - xf[big] * inv) <= np.abs(xf[big] * inv) * 2.0**-4)


def _ref_fixtures():
    import json
    import os

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_gpu_fixtures.json")
    return json.load(open(path))


def test_hash_fill_pinned_to_reference_kernel(orc):
    """kernel_init_stream (src/mem_global.cu:5-12) run on a B200."""
    ref = np.array(_ref_fixtures()["init_stream_4099"], dtype=np.uint32)
    out = np.empty(ref.size, np.uint32)
    orc.orc_fill_hash_u32(ptr(out), out.size)
    assert np.array_equal(out, ref)


def test_chase_walk_pinned_to_reference_kernel(orc):
    """kernel_random_chase_cg (src/memory_chase.cu:29-34) on the oracle's
    4096-slot Sattolo array (seed 0xC0DA): the endpoint after warmup + iters
    hops equals the oracle's walk."""
    links = np.empty(4096 * 32, np.uint32)
    orc.orc_chase_build(ptr(links), links.nbytes, 0xC0DA)
    for case in _ref_fixtures()["chase_cg"]:
        assert orc.orc_chase_walk(ptr(links), case["warmup"] + case["iters"], 0) == case["final"]


def test_constant_mma_sums_pinned_to_reference_kernels():
    """The reference's all-ones mma.sync throughput kernels leave K * iters in
    each accumulator (four per thread, summed); the legacy probes here check
    the same per-accumulator value."""
    fx = _ref_fixtures()
    assert fx["stream_copy_1mib_identical"] is True
    assert fx["hmma_bf16_sum_iters1000"] == 4 * 16 * 1000
    assert fx["hmma_int8_sum_iters1000"] == 4 * 32 * 1000


def test_gemm_tiles_f64_equals_single_tile_oracle(orc):
    """The threaded multi-tile fp64 check sums every element in k order, so
    it equals the single-tile oracle bit for bit (bf16 and e4m3 inputs,
    ragged tile shapes)."""
    rng = np.random.default_rng(5)
    M, N, K = 300, 260, 200
    for dtype in (0, 1):
        if dtype == 0:
            A = (rng.standard_normal(M * K).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
            B = (rng.standard_normal(N * K).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
        else:
            A = rng.integers(0, 0x7f, M * K, dtype=np.uint8)
            B = rng.integers(0, 0x7f, N * K, dtype=np.uint8)
        tiles = np.array([[0, 0, 64, 64], [13, 7, 37, 70], [M - 40, N - 33, 40, 33]], np.int32)
        out = np.zeros(int((tiles[:, 2] * tiles[:, 3]).sum()))
        orc.orc_gemm_tiles_f64(ptr(A), ptr(B), dtype, K, K, K, len(tiles), ptr(tiles), 0.5, 2.0,
                               ptr(out), 3)
        off = 0
        for r0, c0, tm, tn in tiles:
            ref = np.zeros(tm * tn)
            orc.orc_gemm_tile_f64(ptr(A), ptr(B), dtype, K, K, K, int(r0), int(c0), int(tm),
                                  int(tn), 0.5, 2.0, ptr(ref))
            assert np.array_equal(out[off:off + tm * tn], ref), (dtype, r0, c0)
            off += tm * tn
