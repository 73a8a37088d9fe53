"""The softmax of the tcgen05 prefill attention computes a quarter of its
exponentials as 2^x = 2^round(x) * p(x - round(x)) on the FMA pipe (Cody-Waite
range reduction with a fitted degree-5 polynomial, attn_prefill_tc.cu: exp2_poly2).  These
CPU tests replay that arithmetic in float32 with the constants read from the
kernel source and pin its error bound, its bf16 rounding and its edge values."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "qwen3-vl_b200", "csrc", "attn_prefill_tc.cu")


def _coeffs():
    s = open(SRC).read()
    c = [np.float32(float(re.search(rf"kExp2C{i} = ([0-9.e+-]+)f;", s).group(1)))
         for i in (1, 2, 3, 4, 5)]
    return c


def exp2_poly(x):
    """float32 replay of exp2_poly2 (every step rounds to float32 as on the GPU)."""
    c1, c2, c3, c4, c5 = _coeffs()
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-127.0))
    shift = np.float32(12582912.0)
    t = (x + shift).astype(np.float32)
    r = (t + (-shift)).astype(np.float32)
    f = (x - r).astype(np.float32)          # fma(r, -1, x): exact
    q = (f * c5 + c4).astype(np.float32)
    for c in (c3, c2, c1, np.float32(1.0)):
        q = (q * f + c).astype(np.float32)
    bits = q.view(np.int32) + (t.view(np.int32) << np.int32(23))
    return bits.view(np.float32)


def _bf16(v):
    """Round float32 to bf16 (nearest even), returned as float32."""
    u = np.asarray(v, dtype=np.float32).view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def test_relative_error_at_fp32_level():
    # the softmax's arguments: x = s * scale - base <= 8 (lazy rescale)
    x = np.linspace(-125.0, 8.0, 1_000_001).astype(np.float32)
    y = exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() < 2.5e-7, rel.max()


def test_bf16_p_rounds_as_from_the_exact_exponential():
    # P is stored as bf16: the polynomial's keys must round like the exact
    # exponential's (a cubic at 1e-4 changed 5 % of them and flipped near-tie
    # greedy tokens downstream)
    x = np.linspace(-40.0, 8.0, 2_000_001).astype(np.float32)
    got = _bf16(exp2_poly(x))
    want = _bf16(np.exp2(x.astype(np.float64)).astype(np.float32))
    assert np.mean(got != want) < 1e-5


def test_integers_and_edges():
    x = np.arange(-126, 9, dtype=np.float32)
    np.testing.assert_array_equal(exp2_poly(x), np.exp2(x))   # p(0) = 1 exactly
    # masked keys: -inf (and anything at or below -127) give exactly 0
    assert exp2_poly(np.float32(-np.inf)) == 0.0
    assert exp2_poly(np.float32(-127.0)) == 0.0
    assert exp2_poly(np.float32(-1e30)) == 0.0
    # results between 2^-127 and 2^-126 stay tiny and non-negative (ftz-like)
    tiny = exp2_poly(np.linspace(-127.0, -126.0, 101).astype(np.float32))
    assert np.all(tiny >= 0) and np.all(tiny <= np.float32(2.0 ** -125))
    assert np.all(np.isfinite(exp2_poly(np.linspace(-200, 8, 5001).astype(np.float32))))


def test_monotone_on_a_fine_grid():
    # P feeds a sum; a non-monotone approximation would reorder nearly equal keys
    x = np.linspace(-20.0, 0.0, 400_001).astype(np.float32)
    y = exp2_poly(x)
    assert np.all(np.diff(y.astype(np.float64)) >= 0)
