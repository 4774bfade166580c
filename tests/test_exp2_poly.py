"""The FMA-pipe exp2 of the attention softmax (exp2_fma2 in attention.cu),
restated in numpy float32 with the coefficients read from the source: its
relative error stays below f16's half ulp over the range P takes
(x = s * scale - m_ref <= 8), and it underflows cleanly below -30."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(__file__), "..", "ltx-rust_b200", "csrc", "attention.cu")


def coefficients():
    text = open(SRC).read()
    m = re.search(r"constexpr float c0 = ([^,]+), c1 = ([^,]+), c2 = ([^,]+), c3 = ([^;]+);", text)
    assert m, "exp2_fma2 coefficients not found"
    return [np.float32(float.fromhex(v.strip().rstrip("f"))) for v in m.groups()]


def exp2_fma2(x):
    """Float32 restatement: clamp, round-to-nearest split through 1.5 * 2^23, cubic, exponent add."""
    c0, c1, c2, c3 = coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-30.0))
    k = np.float32(12582912.0)
    t = (x + k).astype(np.float32)
    n = (t - k).astype(np.float32)
    f = (x - n).astype(np.float32)
    q = ((c3 * f + c2).astype(np.float32) * f + c1).astype(np.float32)
    q = (q * f + c0).astype(np.float32)
    bits = q.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.view(np.float32)


def test_relative_error_below_f16_half_ulp():
    x = np.linspace(-30.0, 8.0, 2_000_001, dtype=np.float32)
    got = exp2_fma2(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 1.0e-4, rel.max()   # f16 half ulp = 2^-12 = 2.44e-4


def test_clamps_far_below_and_minus_infinity():
    x = np.array([-30.0, -200.0, -1e30, -np.inf], dtype=np.float32)
    got = exp2_fma2(x)
    assert np.all(np.isfinite(got)) and np.all(got > 0) and np.all(got < 2.0 ** -29)
    assert np.all(got.astype(np.float16) == 0)   # rounds to 0 as a P value
