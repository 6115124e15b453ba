"""Property tests of the oracle's number formats and chase builder over
random inputs (hypothesis): the encoders are pinned to their definitions by
brute force, not to a second implementation of the same rounding code."""

import math
import struct

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import ptr

FINITE_E4M3 = [c for c in range(256) if c & 0x7F != 0x7F]


@settings(max_examples=400, deadline=None)
@given(st.floats(width=32, allow_nan=False, allow_infinity=True))
def test_e4m3_satfinite_is_nearest_even(orc, x):
    code = orc.orc_f32_to_e4m3_satfinite(x)
    assert code & 0x7F != 0x7F  # never NaN for a non-NaN input
    got = orc.orc_e4m3_to_f32(code)
    if math.isinf(x) or abs(x) >= 448.0:
        assert got == math.copysign(448.0, x)
        return
    # nearest finite code by exact distance; a tie goes to the even code
    best = min(FINITE_E4M3, key=lambda c: (abs(orc.orc_e4m3_to_f32(c) - x), c & 1))
    assert got == orc.orc_e4m3_to_f32(best), (x, code, best)
    if got == 0.0:
        assert (code >> 7) == (1 if math.copysign(1.0, x) < 0 else 0)


@settings(max_examples=400, deadline=None)
@given(st.floats(width=32, allow_nan=False, allow_infinity=False))
def test_bf16_rne_is_nearest_even(orc, x):
    h = orc.orc_f32_to_bf16_rne(x)
    got = orc.orc_bf16_to_f32(h)
    bits = struct.unpack("<I", struct.pack("<f", x))[0]
    lo, hi = bits & 0xFFFF0000, (bits & 0xFFFF0000) + 0x10000
    down = struct.unpack("<f", struct.pack("<I", lo))[0]
    overflow = (hi & 0x7FFFFFFF) >= 0x7F800000
    if overflow:
        # past the largest finite bf16 the next step is 2^128 with an unbounded
        # exponent; rounding there gives infinity (IEEE 754 overflow rule)
        up_dist = math.copysign(2.0**128, x)
        up = math.copysign(math.inf, x)
    else:
        up = up_dist = struct.unpack("<f", struct.pack("<I", hi & 0xFFFFFFFF))[0]
    dd, du = abs(x - down), abs(up_dist - x)
    if dd < du:
        assert got == down
    elif du < dd:
        assert got == up
    else:
        assert (h & 1) == 0 or overflow  # tie: even mantissa (0x7F80 is even too)
        assert got in (down, up)


@settings(max_examples=60, deadline=None)
@given(st.integers(min_value=1, max_value=5000), st.integers(min_value=0, max_value=2**64 - 1))
def test_chase_builder_single_cycle(orc, slots, seed):
    links = np.empty(slots * 32, np.uint32)
    orc.orc_chase_build(ptr(links), links.nbytes, seed)
    assert orc.orc_chase_is_single_cycle(ptr(links), links.nbytes) == 1
    # slot heads are word indices of slots; padding words are the hash fill
    heads = links[::32]
    assert np.all(heads % 32 == 0) and np.all(heads < slots * 32)
    if slots > 1:
        assert orc.orc_chase_walk(ptr(links), slots, 0) == 0
        assert orc.orc_chase_walk(ptr(links), slots - 1, 0) != 0


@settings(max_examples=40, deadline=None)
@given(st.integers(min_value=1, max_value=24), st.integers(min_value=1, max_value=24),
       st.integers(min_value=1, max_value=80), st.integers(min_value=0, max_value=2**32 - 1))
def test_gemm_tile_f64_against_exact_products(orc, tm, tn, k, seed):
    rng = np.random.default_rng(seed)
    a = rng.integers(0, 256, (tm, k), dtype=np.uint8)
    b = rng.integers(0, 256, (tn, k), dtype=np.uint8)
    a[(a & 0x7F) == 0x7F] = 0  # no NaN codes
    b[(b & 0x7F) == 0x7F] = 0
    out = np.empty((tm, tn), np.float64)
    orc.orc_gemm_tile_f64(ptr(a), ptr(b), 1, k, k, k, 0, 0, tm, tn, 0.5, 2.0, ptr(out))
    dec = np.vectorize(lambda c: orc.orc_e4m3_to_f32(int(c)))
    af, bf = dec(a).astype(np.float64), dec(b).astype(np.float64)
    # e4m3 products and their sums of up to 80 terms are exact in fp64
    ref = np.array([[math.fsum(af[i] * bf[j]) for j in range(tn)] for i in range(tm)])
    assert np.array_equal(out, ref)


@settings(max_examples=60, deadline=None)
@given(st.lists(st.floats(width=32, min_value=-1e6, max_value=1e6), min_size=0, max_size=20000),
       st.integers(min_value=1, max_value=8))
def test_sum_f64_close_to_exact(orc, xs, threads):
    x = np.array(xs, np.float32)
    got = orc.orc_sum_f64(ptr(x) if x.size else 0, x.size, threads)
    exact = math.fsum(float(v) for v in x)
    scale = math.fsum(abs(float(v)) for v in x)
    assert abs(got - exact) <= 1e-12 * max(scale, 1.0)
