"""The MUFU-free tanh used for soft-capped tiles (tanh_poly in
diffuse-rs_b200/csrc/attn_fwd.cuh), replayed in float32 numpy with the
coefficients read from the header, against float64 tanh over the range where
the kernel uses it (|u| <= kTanhPolyMax)."""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "diffuse-rs_b200", "csrc", "attn_fwd.cuh")


def constants():
    src = open(HDR).read()
    c = [1.0]
    for i in range(1, 6):
        m = re.search(rf"kTanhC{i} = ([0-9.e+-]+)f;", src)
        c.append(float(m.group(1)))
    lim = float(re.search(r"kTanhPolyMax = ([0-9.e+-]+)f;", src).group(1))
    return np.array(c, dtype=np.float32), lim


def tanh_poly(u, c):
    u = u.astype(np.float32)
    w = (u * u).astype(np.float32)
    p = np.full_like(w, c[5])
    for i in range(4, -1, -1):
        p = (p * w + c[i]).astype(np.float32)
    return (u * p).astype(np.float32)


def test_error_bound_in_range():
    c, lim = constants()
    u = np.linspace(-lim, lim, 2_000_001).astype(np.float32)
    got = tanh_poly(u, c).astype(np.float64)
    ref = np.tanh(u.astype(np.float64))
    assert np.abs(got - ref).max() < 1e-7
    nz = np.abs(ref) > 1e-6
    assert (np.abs(got[nz] / ref[nz] - 1)).max() < 2.5e-7


def test_odd_and_exact_at_zero():
    c, lim = constants()
    u = np.linspace(0, lim, 1001).astype(np.float32)
    np.testing.assert_array_equal(tanh_poly(-u, c), -tanh_poly(u, c))
    assert tanh_poly(np.zeros(1, np.float32), c)[0] == 0.0
