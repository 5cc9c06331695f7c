"""Pins the CPU oracle (oracle/oracle_attn.c) to the reference's own tests.

Each test restates one reference test (src/model/tests.rs) or checks the
oracle against the committed golden fixtures (tests/golden/), which hold the
reference's modular-ramp inputs and an independent float64 three-pass
softmax. Tolerances are the reference's (1e-5 / 1e-6).
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_cases():
    z = np.load(os.path.join(GOLD, "attention_cases.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    out = {}
    for n in names:
        out[n] = {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")}
    return out


CASES = load_cases()


def run_case(c, kind):
    nq, nk, h, hkv, hd = (int(x) for x in c["dims"])
    win = int(c["window"])
    cp = int(c["causal_prefix"])
    return orc.attention(
        c["q"], c["k"], c["v"], nq=nq, nk=nk, n_head=h, n_head_kv=hkv, head_dim=hd,
        q_pos=c["q_pos"], k_pos=c["k_pos"], q_seq=c.get("qseq"), k_seq=c.get("kseq"),
        q_prefix=c.get("qprefix"), sliding_window=None if win < 0 else win,
        causal_prefix=None if cp < 0 else cp, scale=float(c["scale"]),
        softcap=float(c["softcap"]), kind=kind)


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("kind", [orc.ROW_SCALAR, orc.ROW_AVX2])
def test_oracle_matches_golden(name, kind):
    if kind == orc.ROW_AVX2 and not orc.have_avx2():
        pytest.skip("no AVX2 on this CPU")
    c = CASES[name]
    got = run_case(c, kind)
    np.testing.assert_allclose(got, c["expected"], rtol=0, atol=2e-5, equal_nan=True)


def test_uniform_scores_known_answer():
    # src/model/tests.rs:104-114
    got = run_case(CASES["uniform_scores"], orc.ROW_SCALAR)
    assert abs(got[0] - 2.0) < 1e-6 and abs(got[1] - 4.0) < 1e-6


def test_gqa_matches_repeated_kv():
    # src/model/tests.rs:116-152: GQA 4q/2kv == MHA with kv heads [a,a,b,b].
    c = CASES["gqa_4_2"]
    nq, nk, hd = 3, 5, 8
    k = c["k"].reshape(nk, 2, hd)
    v = c["v"].reshape(nk, 2, hd)
    rep = lambda x: np.repeat(x, 2, axis=1).reshape(-1)  # noqa: E731
    a = orc.attention(c["q"], c["k"], c["v"], nq=nq, nk=nk, n_head=4, n_head_kv=2, head_dim=hd)
    b = orc.attention(c["q"], rep(k), rep(v), nq=nq, nk=nk, n_head=4, n_head_kv=4, head_dim=hd)
    np.testing.assert_allclose(a, b, atol=1e-5, rtol=0)


def test_block_diagonal_equals_separate():
    # src/model/tests.rs:70-102
    c = CASES["block_diag"]
    hd = 4
    batched = run_case(c, orc.ROW_SCALAR)
    q, k, v = c["q"], c["k"], c["v"]
    sa = orc.attention(q[:2 * hd], k[:2 * hd], v[:2 * hd], nq=2, nk=2, n_head=1, n_head_kv=1,
                       head_dim=hd)
    sb = orc.attention(q[2 * hd:], k[2 * hd:], v[2 * hd:], nq=3, nk=3, n_head=1, n_head_kv=1,
                       head_dim=hd)
    np.testing.assert_allclose(batched[:2 * hd], sa, atol=1e-5, rtol=0)
    np.testing.assert_allclose(batched[2 * hd:], sb, atol=1e-5, rtol=0)


def test_avx2_matches_scalar():
    # src/model/tests.rs:188-213
    if not orc.have_avx2():
        pytest.skip("no AVX2")
    for name in ("avx2_hd16", "naive_4x6", "hd320_heap_acc", "window_3"):
        c = CASES[name]
        np.testing.assert_allclose(run_case(c, orc.ROW_AVX2), run_case(c, orc.ROW_SCALAR),
                                   atol=1e-5, rtol=0, equal_nan=True)


def test_all_masked_row_is_nan():
    got = run_case(CASES["all_masked"], orc.ROW_SCALAR)
    assert np.isnan(got).all()


def test_visible_rules():
    # src/model/attention.rs:35-57
    assert not orc.visible(3, 3, 0, 1)
    assert orc.visible(5, 3, 0, 0, window=3)
    assert not orc.visible(6, 3, 0, 0, window=3)
    assert not orc.visible(2, 3, 0, 0, prefix=5)
    assert orc.visible(2, 2, 0, 0, prefix=5)
    assert orc.visible(7, 9, 0, 0, prefix=5)


def test_rope_position_zero_is_identity():
    # src/model/tests.rs:634-640
    rope = orc.build_rope_cache(4, 4, 10000.0)
    x = orc.rotate_rows(np.array([1, 2, 3, 4], np.float32), rope, [0], 1, 4, 4)
    assert x.tolist() == [1.0, 2.0, 3.0, 4.0]


def test_rope_rotates_like_definition():
    rope = orc.build_rope_cache(16, 8, 500000.0).reshape(16, 4, 2)
    x0 = np.arange(16, dtype=np.float32) / 7
    x = orc.rotate_rows(x0, rope.reshape(-1), [9, 3], 1, 8, 8).reshape(2, 8)
    for t, pos in enumerate([9, 3]):
        for i in range(4):
            s, c = rope[pos, i]
            a, b = x0[t * 8 + i], x0[t * 8 + 4 + i]
            assert abs(x[t, i] - (a * c - b * s)) < 1e-6
            assert abs(x[t, 4 + i] - (a * s + b * c)) < 1e-6


def test_cache_store_gather_roundtrip():
    # src/model/tests.rs:55-68
    z = np.load(os.path.join(GOLD, "cache_roundtrip.npz"))
    ck = np.zeros(12, np.float32)
    cv = np.zeros(12, np.float32)
    orc.cache_store(ck, cv, 4, z["store_pos"], z["k"], z["v"])
    ok, ov = orc.cache_gather(ck, cv, 4, z["gather_pos"])
    assert ok.tolist() == z["out_k"].tolist()
    assert ov.tolist() == z["out_v"].tolist()


def test_rms_norm_matches_f64_definition():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(128).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    got = orc.rms_norm_inplace(x.copy(), w, 1e-6)
    ss = float(np.sum((x * x).astype(np.float64)))
    sc = np.float32(1.0) / np.float32(np.sqrt(ss / 128 + 1e-6))
    want = (x * sc) * w
    np.testing.assert_array_equal(got, want)


def test_oracle_threads_do_not_change_results():
    c = CASES["hd320_heap_acc"]
    nq, nk, h, hkv, hd = (int(x) for x in c["dims"])
    a = orc.attention(c["q"], c["k"], c["v"], nq=nq, nk=nk, n_head=h, n_head_kv=hkv,
                      head_dim=hd, threads=1)
    b = orc.attention(c["q"], c["k"], c["v"], nq=nq, nk=nk, n_head=h, n_head_kv=hkv,
                      head_dim=hd, threads=8)
    np.testing.assert_array_equal(a, b)
