"""ctypes wrapper over liboracle_attn.so, the CPU restatement of diffuse-rs
canvas attention.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker or the timed CPU
baseline -- never by the product package.

Every function mirrors one reference function; the C source cites the
reference file:line for each (src/model/attention.rs, src/model/ops.rs,
src/model/cache.rs, src/model/sampler.rs, src/kernels.rs, src/model/matmul.rs).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_attn.so")

ROW_SCALAR = 0
ROW_AVX2 = 1


class OrShape(ctypes.Structure):
    _fields_ = [
        ("nq", ctypes.c_int64),
        ("nk", ctypes.c_int64),
        ("n_head", ctypes.c_int64),
        ("n_head_kv", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("sliding_window", ctypes.c_int64),
        ("causal_prefix", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("softcap", ctypes.c_float),
    ]


class OrRows(ctypes.Structure):
    _fields_ = [
        ("pos", ctypes.POINTER(ctypes.c_int64)),
        ("seq", ctypes.POINTER(ctypes.c_int64)),
        ("n_seq", ctypes.c_int64),
        ("prefix", ctypes.POINTER(ctypes.c_int64)),
        ("n_prefix", ctypes.c_int64),
    ]


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        ip = ctypes.POINTER(ctypes.c_int64)
        L.or_attention.argtypes = [fp, fp, fp, fp, ctypes.POINTER(OrShape),
                                   ctypes.POINTER(OrRows), ctypes.POINTER(OrRows),
                                   ctypes.c_int, ctypes.c_int]
        L.or_attention.restype = ctypes.c_int
        L.or_attention_tasks.argtypes = [fp, fp, fp, fp, ctypes.POINTER(OrShape),
                                         ctypes.POINTER(OrRows), ctypes.POINTER(OrRows),
                                         ip, ctypes.c_int64, ctypes.c_int, ctypes.c_int]
        L.or_attention_tasks.restype = ctypes.c_int
        L.or_visible.argtypes = [ctypes.c_int64] * 6
        L.or_visible.restype = ctypes.c_int
        L.or_rms_norm_inplace.argtypes = [fp, fp, ctypes.c_int64, ctypes.c_float]
        L.or_rms_norm_noscale.argtypes = [fp, ctypes.c_int64, ctypes.c_float]
        L.or_norm_heads.argtypes = [fp, ctypes.c_int64, fp, ctypes.c_int64, ctypes.c_float]
        L.or_build_rope_cache.argtypes = [fp, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_float, fp]
        L.or_rotate_rows.argtypes = [fp, fp, ip, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_int64]
        L.or_cache_store.argtypes = [fp, fp, ctypes.c_int64, ip, ctypes.c_int64, fp, fp]
        L.or_cache_gather.argtypes = [fp, fp, ctypes.c_int64, ip, ctypes.c_int64, fp, fp]
        i32p = ctypes.POINTER(ctypes.c_int32)
        L.or_compute_entropy.argtypes = [fp, ctypes.c_int64]
        L.or_compute_entropy.restype = ctypes.c_float
        L.or_log_sum_exp.argtypes = [fp, ctypes.c_int64]
        L.or_log_sum_exp.restype = ctypes.c_float
        L.or_top2_logits.argtypes = [fp, ctypes.c_int64, fp, fp]
        L.or_pick_greedy.argtypes = [fp, ctypes.c_int64]
        L.or_pick_greedy.restype = ctypes.c_int32
        L.or_candidate_stats.argtypes = [fp, ctypes.c_int64, ctypes.c_int64, i32p,
                                         ctypes.c_int64, ctypes.c_int32, i32p, ctypes.c_int64,
                                         ctypes.c_int, ctypes.c_int, i32p, fp, fp, fp]
        L.or_tokens_to_unmask.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_int32]
        L.or_tokens_to_unmask.restype = ctypes.c_int64
        u8p = ctypes.POINTER(ctypes.c_uint8)
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_dequant_row.argtypes = [ctypes.c_int32, u8p, ctypes.c_int64, fp]
        L.or_dequant_row.restype = ctypes.c_int
        L.or_row_bytes.argtypes = [ctypes.c_int32, ctypes.c_int64]
        L.or_row_bytes.restype = ctypes.c_int64
        L.or_quantize_row_q8k.argtypes = [fp, ctypes.c_int64, fp, ctypes.POINTER(ctypes.c_int8),
                                          ctypes.POINTER(ctypes.c_int16)]
        L.or_vec_dot_q4k_q8k.argtypes = [u8p, fp, ctypes.POINTER(ctypes.c_int8),
                                         ctypes.POINTER(ctypes.c_int16), ctypes.c_int64]
        L.or_vec_dot_q4k_q8k.restype = ctypes.c_float
        L.or_vec_dot_q6k_q8k.argtypes = [u8p, fp, ctypes.POINTER(ctypes.c_int8), ctypes.c_int64]
        L.or_vec_dot_q6k_q8k.restype = ctypes.c_float
        L.or_linear_q8k.argtypes = [ctypes.c_int32, u8p, ctypes.c_int64, ctypes.c_int64, fp,
                                    ctypes.c_int64, fp]
        L.or_linear_q8k.restype = ctypes.c_int
        L.or_have_avx2.restype = ctypes.c_int
        L.or_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _i64(a):
    if a is None or len(a) == 0:
        return None, None, 0
    a = np.ascontiguousarray(a, dtype=np.int64)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), len(a)


def _rows(pos, seq=None, prefix=None):
    keep = []
    p, pp, _ = _i64(pos)
    s, sp, ns = _i64(seq)
    f, fp, nf = _i64(prefix)
    keep += [p, s, f]
    r = OrRows(pp, sp, ns, fp, nf)
    return r, keep


def attention(q, k, v, *, nq, nk, n_head, n_head_kv, head_dim,
              q_pos=None, k_pos=None, q_seq=None, k_seq=None, q_prefix=None,
              sliding_window=None, causal_prefix=None, scale=1.0, softcap=0.0,
              kind=ROW_SCALAR, threads=0, tasks=None, out=None):
    """attention() over fp32 numpy buffers laid out as in the reference.

    Positions default to 0..n-1 (the reference's idpos helper in its tests).
    """
    L = lib()
    q, qp = _f32(q)
    k, kp = _f32(k)
    v, vp = _f32(v)
    if out is None:
        out = np.zeros(nq * n_head * head_dim, dtype=np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    op = out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    if q_pos is None:
        q_pos = np.arange(nq, dtype=np.int64)
    if k_pos is None:
        k_pos = np.arange(nk, dtype=np.int64)
    s = OrShape(nq, nk, n_head, n_head_kv, head_dim,
                -1 if sliding_window is None else int(sliding_window),
                -1 if causal_prefix is None else int(causal_prefix),
                float(scale), float(softcap))
    qr, kq = _rows(q_pos, q_seq, q_prefix)
    kr, kk = _rows(k_pos, k_seq, None)
    if tasks is None:
        rc = L.or_attention(op, qp, kp, vp, ctypes.byref(s), ctypes.byref(qr),
                            ctypes.byref(kr), kind, threads)
    else:
        t, tp, nt = _i64(tasks)
        rc = L.or_attention_tasks(op, qp, kp, vp, ctypes.byref(s), ctypes.byref(qr),
                                  ctypes.byref(kr), tp, nt, kind, threads)
    if rc != 0:
        raise RuntimeError(f"oracle attention failed: {rc}")
    return out


def visible(qpos, kpos, qseq, kseq, window=None, prefix=None):
    return bool(lib().or_visible(qpos, kpos, qseq, kseq,
                                 -1 if window is None else window,
                                 -1 if prefix is None else prefix))


def rms_norm_inplace(x, w, eps):
    x, xp = _f32(x)
    w, wp = _f32(w)
    lib().or_rms_norm_inplace(xp, wp, len(x), eps)
    return x


def norm_heads(x, w, eps):
    x = np.array(x, dtype=np.float32, copy=True).reshape(-1)
    _, xp = _f32(x)
    w, wp = _f32(w)
    lib().or_norm_heads(xp, len(x), wp, len(w), eps)
    return x


def rms_norm_noscale(x, eps):
    x = np.array(x, dtype=np.float32, copy=True).reshape(-1)
    _, xp = _f32(x)
    lib().or_rms_norm_noscale(xp, len(x), eps)
    return x


def build_rope_cache(max_seq_len, rope_dim, theta, freq_factors=None):
    out = np.zeros(max_seq_len * (rope_dim // 2) * 2, dtype=np.float32)
    _, op = _f32(out)
    ff = None
    if freq_factors is not None:
        ffa, ff = _f32(freq_factors)
    lib().or_build_rope_cache(op, max_seq_len, rope_dim, theta, ff)
    return out


def rotate_rows(x, rope, positions, heads, hd, rot):
    x = np.array(x, dtype=np.float32, copy=True).reshape(-1)
    _, xp = _f32(x)
    rope, rp = _f32(rope)
    pos, pp, n = _i64(positions)
    lib().or_rotate_rows(xp, rp, pp, n, heads, hd, rot)
    return x


def cache_store(cache_k, cache_v, stride, positions, k, v):
    assert cache_k.dtype == np.float32 and cache_v.dtype == np.float32
    ck = cache_k.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    cv = cache_v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    k, kp = _f32(k)
    v, vp = _f32(v)
    pos, pp, n = _i64(positions)
    lib().or_cache_store(ck, cv, stride, pp, n, kp, vp)


def cache_gather(cache_k, cache_v, stride, positions):
    ck, ckp = _f32(cache_k)
    cv, cvp = _f32(cache_v)
    pos, pp, n = _i64(positions)
    ok = np.zeros(n * stride, dtype=np.float32)
    ov = np.zeros(n * stride, dtype=np.float32)
    lib().or_cache_gather(ckp, cvp, stride, pp, n,
                          ok.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                          ov.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return ok, ov


def have_avx2() -> bool:
    return bool(lib().or_have_avx2())


def max_threads() -> int:
    return int(lib().or_max_threads())


# ---------------------------------------------------------------- sampler
def compute_entropy(row):
    row, rp = _f32(row)
    return float(lib().or_compute_entropy(rp, len(row)))


def log_sum_exp(row):
    row, rp = _f32(row)
    return float(lib().or_log_sum_exp(rp, len(row)))


def top2_logits(row):
    row, rp = _f32(row)
    t1, t2 = ctypes.c_float(), ctypes.c_float()
    lib().or_top2_logits(rp, len(row), ctypes.byref(t1), ctypes.byref(t2))
    return float(t1.value), float(t2.value)


def candidate_stats(logits, rows, *, mask_id=-1, suppress=(), want_entropy=True,
                    want_prob=True):
    """collect_candidates' per-row statistics (greedy pick) on a copy of
    `logits` [rows_total, n_vocab]; returns (token, entropy, margin, prob)."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    n_rows, n_vocab = lg.shape
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    sup = np.ascontiguousarray(suppress, dtype=np.int32)
    n = len(rows)
    tok = np.zeros(n, np.int32)
    ent, mar, prob = (np.zeros(n, np.float32) for _ in range(3))
    i32p = ctypes.POINTER(ctypes.c_int32)
    fp = ctypes.POINTER(ctypes.c_float)
    lib().or_candidate_stats(lg.ctypes.data_as(fp), n_rows, n_vocab, rows.ctypes.data_as(i32p),
                             n, int(mask_id), sup.ctypes.data_as(i32p), len(sup),
                             int(want_entropy), int(want_prob), tok.ctypes.data_as(i32p),
                             ent.ctypes.data_as(fp), mar.ctypes.data_as(fp),
                             prob.ctypes.data_as(fp))
    return tok, ent, mar, prob


def tokens_to_unmask(step, total_steps, masked, schedule):
    """schedule: 0 cosine, 1 linear (src/model/sampler.rs:115-132)."""
    return int(lib().or_tokens_to_unmask(step, total_steps, masked, schedule))


# ---------------------------------------------------------------- quantised weights
QTYPE_F16, QTYPE_Q4_0, QTYPE_Q8_0, QTYPE_Q4_K, QTYPE_Q6_K = 1, 2, 8, 12, 14


def _u8(a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def f16_to_f32(h):
    return float(lib().or_f16_to_f32(int(h)))


def row_bytes(qtype, cols):
    return int(lib().or_row_bytes(int(qtype), int(cols)))


def dequantize(qtype, w_bytes, rows, cols):
    """[rows, cols] f32 from `rows` rows of `cols` weights of type qtype."""
    w, wp = _u8(w_bytes)
    rb = row_bytes(qtype, cols)
    out = np.zeros((rows, cols), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    for r in range(rows):
        rc = lib().or_dequant_row(int(qtype), ctypes.cast(ctypes.addressof(wp.contents) + r * rb,
                                                           ctypes.POINTER(ctypes.c_uint8)),
                                  int(cols), out[r].ctypes.data_as(fp))
        if rc != 0:
            raise ValueError(f"unknown qtype {qtype}")
    return out


def quantize_row_q8k(x):
    x, xp = _f32(x)
    nb = len(x) // 256
    d = np.zeros(nb, np.float32)
    qs = np.zeros(nb * 256, np.int8)
    bs = np.zeros(nb * 16, np.int16)
    lib().or_quantize_row_q8k(xp, nb, d.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                              qs.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)),
                              bs.ctypes.data_as(ctypes.POINTER(ctypes.c_int16)))
    return d, qs, bs


def vec_dot_q4k_q8k(w_bytes, d, qs, bs):
    w, wp = _u8(w_bytes)
    return float(lib().or_vec_dot_q4k_q8k(wp, _f32(d)[1], qs.ctypes.data_as(
        ctypes.POINTER(ctypes.c_int8)), bs.ctypes.data_as(ctypes.POINTER(ctypes.c_int16)),
        len(d)))


def vec_dot_q6k_q8k(w_bytes, d, qs):
    w, wp = _u8(w_bytes)
    return float(lib().or_vec_dot_q6k_q8k(wp, _f32(d)[1], qs.ctypes.data_as(
        ctypes.POINTER(ctypes.c_int8)), len(d)))


def linear_q8k(qtype, w_bytes, rows, cols, act):
    """The reference's Q4_K / Q6_K projection (activations quantised to
    Q8_K): [n, rows] f32 for act [n, cols]."""
    w, wp = _u8(w_bytes)
    act = np.ascontiguousarray(act, dtype=np.float32)
    n = act.shape[0]
    out = np.zeros((n, rows), np.float32)
    rc = lib().or_linear_q8k(int(qtype), wp, int(rows), int(cols),
                             act.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n,
                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    if rc != 0:
        raise ValueError("or_linear_q8k: unsupported type or width")
    return out
