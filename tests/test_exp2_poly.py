"""The FMA-pipe exp2 used by the softmax (ex2_poly in
diffuse-rs_b200/csrc/sm100.cuh), replayed in float32 numpy with the
coefficients read from the header, against float64 exp2."""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "diffuse-rs_b200", "csrc", "sm100.cuh")


def coeffs():
    src = open(HDR).read()
    c = [1.0]
    for i in range(1, 6):
        m = re.search(rf"kExp2C{i} = ([0-9.e+-]+)f;", src)
        c.append(float(m.group(1)))
    return np.array(c, dtype=np.float32)


def ex2_poly(x, c):
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    f = (x - (t - np.float32(12582912.0))).astype(np.float32)
    p = c[5]
    for i in range(4, -1, -1):
        p = (p * f + c[i]).astype(np.float32)
    n = t.view(np.int32) - np.int32(0x4B400000)
    return (p.view(np.int32) + (n << 23)).view(np.float32)


def test_relative_error_bound():
    c = coeffs()
    x = np.linspace(-126, 8, 1_000_001).astype(np.float32)
    got = ex2_poly(x, c).astype(np.float64)
    rel = np.abs(got / np.exp2(x.astype(np.float64)) - 1)
    assert rel.max() < 2.5e-7, rel.max()


def test_exact_at_integers_and_clamped_below():
    c = coeffs()
    x = np.arange(-126, 9, dtype=np.float32)
    np.testing.assert_array_equal(ex2_poly(x, c), np.exp2(x))
    assert ex2_poly(np.array([-1e9], np.float32), c)[0] == np.float32(2.0 ** -126)
