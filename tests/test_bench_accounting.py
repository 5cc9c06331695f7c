"""The work accounting behind every number bench.py reports (CPU only).

FLOPs = 4 * head_dim * visible (query, key) pairs * n_head over the batch
and layers; visible pairs follow visible() (src/model/attention.rs:35-57):
|q pos - k pos| < window when a window is set. Bytes = one bf16 read of Q, K,
V and one bf16 write of O."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("na,n_total,start,window", [
    (64, 64, 0, None), (64, 64, 0, 1), (64, 64, 0, 7), (100, 300, 150, 20),
    (32, 4128, 2048, None), (257, 257, 0, 512), (300, 300, 0, 64)])
def test_visible_pairs_matches_brute_force(na, n_total, start, window):
    brute = sum(1 for q in range(start, start + na) for k in range(n_total)
                if window is None or abs(q - k) < window)
    assert bench.visible_pairs(na, n_total, start, window) == brute


def test_step_flops_of_the_configs():
    # GFLOP per step: 4 * hd * visible pairs * H * B, summed over layers.
    want = {"c1": 0.268435456, "c2": 60.129542144, "c3": 1099.511627776,
            "c4": 34.628173824}
    for c, g in want.items():
        assert bench.step_flops(bench.CONFIGS[c]) / 1e9 == pytest.approx(g, rel=1e-12)
    c5 = bench.CONFIGS["c5"]
    glob = bench.layer_flops(c5, None) / 1e9
    slide = bench.layer_flops(c5, 512) / 1e9
    assert glob == pytest.approx(4398.046511104, rel=1e-12)
    # 8192 queries, each seeing min(8191, q + 511) - max(0, q - 511) + 1 keys.
    pairs = sum(min(8191, q + 511) - max(0, q - 511) + 1 for q in range(8192))
    assert slide == pytest.approx(4 * 256 * 16 * 4 * pairs / 1e9, rel=1e-12)
    assert bench.step_flops(c5) / 1e9 == pytest.approx(glob + 5 * slide, rel=1e-12)


def test_layer_bytes_of_the_configs():
    mb = {c: bench.layer_bytes(bench.CONFIGS[c]) / 1e6 for c in ("c2", "c3", "c4")}
    assert mb["c3"] == pytest.approx(536.870912)  # 402.7 read + 134.2 write
    assert mb["c2"] == pytest.approx(67.108864)
    assert mb["c4"] == pytest.approx(278.921216)  # cache 270.5 MB + Q + O
