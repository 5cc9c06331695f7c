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


def poly3_coeffs():
    src = open(HDR).read()
    return [np.float32(float(re.search(rf"kExp2D{i} = ([0-9.e+-]+)f;", src).group(1)))
            for i in (1, 2, 3)]


def ex2_poly3x2(x, c):
    """float32 replay of ex2_poly3x2 (sm100.cuh) on one lane."""
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    tm = (t + np.float32(-12582912.0)).astype(np.float32)
    f = (x - tm).astype(np.float32)
    p = (c[2] * f + c[1]).astype(np.float32)
    p = (p * f + c[0]).astype(np.float32)
    p = (p * f + np.float32(1.0)).astype(np.float32)
    return (p.view(np.int32) + (t.view(np.int32) << 23)).view(np.float32)


def test_degree3_exp2_error_bound_below_bf16_rounding():
    # The softmax weights it produces are rounded to bf16 (relative step
    # 2^-8); the stated bound is 1.0e-4 on the range softmax logits take.
    x = np.linspace(-20.0, 8.0, 1_400_001).astype(np.float32)
    got = ex2_poly3x2(x, poly3_coeffs()).astype(np.float64)
    rel = np.abs(got / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 1.1e-4
    # Very negative inputs clamp to 2^-126, never wrap.
    y = ex2_poly3x2(np.array([-126.0, -200.0, -1e30], np.float32), poly3_coeffs())
    assert np.all(y > 0) and np.all(y < 1.2e-38)
