"""Generate the golden fixtures that pin the CPU oracle (tests/golden/*.npz).

Inputs are the reference's own deterministic modular ramps
(src/model/tests.rs:80-82, :124-128, :159-161, :195-198) at the reference's own
test shapes, plus build-authored cases for semantics the reference leaves
untested (sliding window, causal prefix, per-row prefix, scale != 1,
head_dim > 256, fully-masked rows, reordered cached keys, soft-cap extension).

Expected outputs come from an independent float64 three-pass softmax written
here in numpy -- the same "naive reference" the reference's
test_attention_matches_naive_reference uses (src/model/tests.rs:154-186 with
softmax_row_scalar, src/model/ops.rs:269-280) -- with visible() restated from
src/model/attention.rs:35-57. It shares no code with oracle/oracle_attn.c.

The Rust reference cannot run in this container (no cargo/rustc), so these
fixtures plus the reference's known answers ([2, 4] at tests.rs:104-114, the
cache layout at tests.rs:55-68, RoPE identity at tests.rs:634-640) are the
pins. Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def ramp(n, mul, mod, off, div):
    """((x * mul % mod) - off) / div as f32, the reference's test generator."""
    x = np.arange(n, dtype=np.int64)
    return (((x * mul) % mod).astype(np.float32) - np.float32(off)) / np.float32(div)


def visible(qpos, kpos, qseq, kseq, window, prefix):
    if qseq != kseq:
        return False
    if window is not None and abs(qpos - kpos) >= window:
        return False
    if prefix is not None and qpos < prefix:
        return kpos <= qpos
    return True


def naive(q, k, v, nq, nk, h, hkv, hd, qpos, kpos, qseq=None, kseq=None,
          qprefix=None, window=None, causal_prefix=None, scale=1.0, softcap=0.0):
    q = q.astype(np.float64).reshape(nq, h, hd)
    k = k.astype(np.float64).reshape(nk, hkv, hd)
    v = v.astype(np.float64).reshape(nk, hkv, hd)
    out = np.zeros((nq, h, hd))
    g = h // hkv
    for head in range(h):
        kvh = head // g
        for i in range(nq):
            pre = causal_prefix if qprefix is None else qprefix[i]
            qs = 0 if qseq is None else qseq[i]
            vis = [j for j in range(nk)
                   if visible(qpos[i], kpos[j], qs, 0 if kseq is None else kseq[j],
                              window, pre)]
            if not vis:
                out[i, head] = np.nan  # sum == 0: acc * (1/0) = 0 * inf
                continue
            s = np.array([q[i, head] @ k[j, kvh] for j in vis]) * scale
            if softcap > 0:
                s = softcap * np.tanh(s / softcap)
            p = np.exp(s - s.max())
            p /= p.sum()
            out[i, head] = p @ v[vis, kvh]
    return out.reshape(-1).astype(np.float32)


def case(name, nq, nk, h, hkv, hd, q, k, v, qpos=None, kpos=None, **kw):
    qpos = list(range(nq)) if qpos is None else list(qpos)
    kpos = list(range(nk)) if kpos is None else list(kpos)
    exp = naive(q, k, v, nq, nk, h, hkv, hd, qpos, kpos, **kw)
    d = dict(q=q, k=k, v=v, expected=exp,
             dims=np.array([nq, nk, h, hkv, hd], np.int64),
             q_pos=np.array(qpos, np.int64), k_pos=np.array(kpos, np.int64),
             scale=np.float32(kw.get("scale", 1.0)),
             softcap=np.float32(kw.get("softcap", 0.0)),
             window=np.int64(-1 if kw.get("window") is None else kw["window"]),
             causal_prefix=np.int64(-1 if kw.get("causal_prefix") is None
                                    else kw["causal_prefix"]))
    for key in ("qseq", "kseq", "qprefix"):
        if kw.get(key) is not None:
            d[key] = np.array(kw[key], np.int64)
    return name, d


def all_cases():
    cs = []
    # tests.rs:104-114 known answer: identical keys -> mean of V = [2, 4].
    cs.append(case("uniform_scores", 1, 2, 1, 1, 2,
                   np.array([1, 0], np.float32), np.array([1, 0, 1, 0], np.float32),
                   np.array([0, 2, 4, 6], np.float32)))
    # tests.rs:116-152 GQA 4q/2kv shapes and ramps.
    nq, nk, hd = 3, 5, 8
    cs.append(case("gqa_4_2", nq, nk, 4, 2, hd, ramp(nq * 4 * hd, 37, 101, 50, 50),
                   ramp(nk * 2 * hd, 53, 97, 48, 48), ramp(nk * 2 * hd, 71, 89, 44, 44)))
    # tests.rs:154-186 online vs naive.
    cs.append(case("naive_4x6", 4, 6, 2, 2, 8, ramp(4 * 2 * 8, 37, 101, 50, 25),
                   ramp(6 * 2 * 8, 53, 97, 48, 24), ramp(6 * 2 * 8, 71, 89, 44, 44)))
    # tests.rs:70-102 block-diagonal batch: seq ids [0,0,1,1,1], pos [0,1,0,1,2].
    q = ramp(5 * 4, 37, 101, 50, 50)
    cs.append(case("block_diag", 5, 5, 1, 1, 4, q, q.copy(), ramp(5 * 4, 71, 89, 44, 44),
                   qpos=[0, 1, 0, 1, 2], kpos=[0, 1, 0, 1, 2],
                   qseq=[0, 0, 1, 1, 1], kseq=[0, 0, 1, 1, 1]))
    # tests.rs:188-213 AVX2 vs scalar shape (hd 16).
    n = 3 * 2 * 16
    cs.append(case("avx2_hd16", 3, 3, 2, 2, 16, ramp(n, 37, 101, 50, 50),
                   ramp(n, 53, 97, 48, 48), ramp(n, 71, 89, 44, 44)))
    # Build-authored KATs (not pinned by the reference's tests).
    rng = np.random.default_rng(1234)

    def rnd(*s):
        return rng.standard_normal(int(np.prod(s))).astype(np.float32)

    cs.append(case("window_3", 12, 12, 2, 1, 16, rnd(12, 2, 16), rnd(12, 16), rnd(12, 16),
                   window=3, scale=0.25))
    cs.append(case("causal_prefix_5", 10, 10, 2, 2, 8, rnd(10, 2, 8), rnd(10, 2, 8),
                   rnd(10, 2, 8), causal_prefix=5, scale=0.35))
    cs.append(case("row_prefix", 7, 7, 1, 1, 8, rnd(7, 8), rnd(7, 8), rnd(7, 8),
                   qprefix=[3, 3, 3, 0, 6, 6, 2], scale=0.5))
    cs.append(case("hd320_heap_acc", 4, 9, 2, 1, 320, rnd(4, 2, 320), rnd(9, 320),
                   rnd(9, 320), scale=320 ** -0.5))
    # Fully masked row: window 0 hides every key -> NaN (0 * 1/0).
    cs.append(case("all_masked", 2, 3, 1, 1, 4, rnd(2, 4), rnd(3, 4), rnd(3, 4), window=0))
    # Cached path: keys are [cached asc | active asc] (forward.rs:92-96).
    cached = [0, 1, 4, 5, 7]
    active = [2, 3, 6]
    cs.append(case("cached_reorder", 3, 8, 4, 2, 16, rnd(3, 4, 16), rnd(8, 2, 16),
                   rnd(8, 2, 16), qpos=active, kpos=cached + active, window=3,
                   scale=0.25))
    cs.append(case("softcap_ext", 5, 11, 2, 2, 8, rnd(5, 2, 8) * 4, rnd(11, 2, 8) * 4,
                   rnd(11, 2, 8), softcap=5.0, scale=1.0))
    return cs


def main():
    cs = all_cases()
    arrays = {}
    for name, d in cs:
        for key, val in d.items():
            arrays[f"{name}/{key}"] = val
    np.savez_compressed(os.path.join(HERE, "attention_cases.npz"), **arrays)

    # tests.rs:55-68 cache store/gather round trip (exact expected values).
    k = np.arange(8, dtype=np.float32)
    v = k + 100
    np.savez_compressed(
        os.path.join(HERE, "cache_roundtrip.npz"),
        k=k, v=v, store_pos=np.array([2, 0], np.int64), gather_pos=np.array([0, 2], np.int64),
        out_k=np.array([4, 5, 6, 7, 0, 1, 2, 3], np.float32),
        out_v=np.array([104, 105, 106, 107, 100, 101, 102, 103], np.float32))
    print(f"wrote {len(cs)} attention cases")


if __name__ == "__main__":
    main()
