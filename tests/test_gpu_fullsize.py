"""Parity at BASELINE.json's full sizes, through the entry point bench.py
times (default single-term softmax weights; fp32 output so that the 2e-3 bar
applies to the attention itself, not to a final bf16 rounding).

Rows of attention are independent (src/model/attention.rs:116 runs each
(head, query) as its own task), so a seeded sample of rows checked against the
oracle is an exact check of those rows; c2 and c4 are small enough to check
whole sequences. Also: the same call twice gives bit-identical output."""
import numpy as np
import pytest
import torch

import canvas_attn as ca
from helpers import bf16_round, check_close
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _block(cfg_seed, B, na, n_total, start, H, Hkv, hd, theta, qk_norm, window=None,
           softcap=0.0, scale=None, precise=False):
    """Runs one fused block on the GPU; returns inputs (fp32 CPU) and output."""
    g = torch.Generator().manual_seed(cfg_seed)
    scale = hd ** -0.5 if scale is None else scale
    q = bf16_round(torch.randn(B, na, H, hd, generator=g))
    k = bf16_round(torch.randn(B, na, Hkv, hd, generator=g))
    v = bf16_round(torch.randn(B, na, Hkv, hd, generator=g))
    cache_k = bf16_round(torch.randn(B, n_total, Hkv, hd, generator=g))
    cache_v = bf16_round(torch.randn(B, n_total, Hkv, hd, generator=g))
    wq = (torch.rand(hd, generator=g) + 0.5) if qk_norm else None
    wk = (torch.rand(hd, generator=g) + 0.5) if qk_norm else None
    rope = ca.build_rope_cache(max(4096, n_total), hd, theta)
    pos = torch.arange(start, start + na, dtype=torch.int32).repeat(B, 1)
    dk = cache_k.to(torch.bfloat16).cuda()
    dv = cache_v.to(torch.bfloat16).cuda()
    out = torch.empty(B, na, H, hd, dtype=torch.float32, device="cuda")
    q_work = torch.empty(B, na, H, hd, dtype=torch.bfloat16, device="cuda")
    args = dict(batch=B, n_active=na, active_pos=pos.cuda(), rope=torch.from_numpy(rope).cuda(),
                rope_len=max(4096, n_total), rope_dim=hd, cache_k=dk, cache_v=dv,
                n_total=n_total, q_work=q_work, out=out, n_head=H, n_head_kv=Hkv, head_dim=hd,
                q_norm_w=None if wq is None else wq.cuda(),
                k_norm_w=None if wk is None else wk.cuda(), rms_eps=1e-6,
                out_f32=True, sliding_window=window, scale=scale, softcap=softcap,
                precise=precise)
    dq, dk_in, dv_in = (x.to(torch.bfloat16).cuda() for x in (q, k, v))
    ca.attention_block_dev(dq, dk_in, dv_in, **args)
    torch.cuda.synchronize()
    first = out.clone()
    ca.attention_block_dev(dq, dk_in, dv_in, **args)  # cache now holds these K/V again
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    assert torch.equal(first, out), "repeated call is not bit-identical"
    return dict(q=q, k=k, v=v, cache_k=dk.float().cpu(), cache_v=dv.float().cpu(), wq=wq,
                wk=wk, rope=rope, pos=np.arange(start, start + na), out=out.float().cpu(),
                B=B, na=na, n_total=n_total, H=H, Hkv=Hkv, hd=hd, scale=scale,
                window=window, softcap=softcap)


def _oracle_seq(d, b, tasks=None):
    """Oracle for sequence b: pre-ops in fp32 on the bf16 inputs, post-RoPE Q
    rounded to bf16 (the attention operands are bf16); keys = the GPU's cache
    after the store (active rows at their positions), all positions."""
    H, Hkv, hd, na = d["H"], d["Hkv"], d["hd"], d["na"]
    q = d["q"][b].numpy().reshape(-1)
    if d["wq"] is not None:
        q = orc.norm_heads(q, d["wq"].numpy(), 1e-6)
    q = orc.rotate_rows(q, d["rope"], d["pos"], H, hd, hd)
    q = bf16_round(torch.from_numpy(q)).numpy()
    kf = d["cache_k"][b].numpy().reshape(-1)
    vf = d["cache_v"][b].numpy().reshape(-1)
    out = orc.attention(q, kf, vf, nq=na, nk=d["n_total"], n_head=H, n_head_kv=Hkv,
                        head_dim=hd, q_pos=d["pos"], k_pos=np.arange(d["n_total"]),
                        sliding_window=d["window"], scale=d["scale"], softcap=d["softcap"],
                        kind=orc.ROW_AVX2 if orc.have_avx2() else orc.ROW_SCALAR,
                        tasks=tasks)
    return out.reshape(na, H, hd)


def _check_rows(d, b, n_rows, seed, atol=2e-3):
    """Sampled rows, per-element 2e-3 and rel-L2 1e-2."""
    rng = np.random.default_rng(seed)
    H, na, hd = d["H"], d["na"], d["hd"]
    tasks = np.sort(rng.choice(H * na, size=n_rows, replace=False)).astype(np.int64)
    ref = _oracle_seq(d, b, tasks)
    got = d["out"][b].numpy()
    heads, rows = tasks // na, tasks % na
    g = got[rows, heads]
    r = ref[rows, heads]
    check_close(g.reshape(-1, 1, hd), r.reshape(-1, 1, hd), 1, hd, atol=atol, rel=1e-2,
                what=f"seq {b}")


def test_c3_fullsize_rows():
    d = _block(3, 8, 4096, 4096, 0, 16, 16, 128, 5e4, True)
    for b in (0, 5):
        _check_rows(d, b, 256, seed=b)


def test_c4_fullsize_sequences():
    d = _block(4, 16, 32, 4128, 2048, 32, 8, 128, 5e5, False)
    for b in (0, 9, 15):
        ref = _oracle_seq(d, b)
        check_close(d["out"][b].numpy(), ref, 32, 128, what=f"c4 seq {b}")


def test_c2_fullsize_sequence():
    d = _block(2, 4, 1024, 1024, 0, 28, 4, 128, 1e6, False)
    ref = _oracle_seq(d, 2)
    check_close(d["out"][2].numpy(), ref, 28, 128, what="c2 seq 2")


@pytest.mark.parametrize("window,theta", [(512, 1e4), (None, 1e6)])
def test_c5_fullsize_rows(window, theta):
    d = _block(5, 4, 8192, 8192, 0, 16, 8, 256, theta, True, window=window, softcap=50.0,
               scale=256 ** -0.5)
    _check_rows(d, 1, 128, seed=7)


def test_gemma_global_layer_head_dim_512_fullsize_rows():
    # c5's shape with the real DiffusionGemma global-layer heads: B4 S8192,
    # 16 query heads over 2 kv heads (GQA group 8), head_dim 512, QK-norm,
    # soft-cap 50, scale 1.0 (forward.rs:341). With scale 1.0 the normed
    # scores reach the soft-cap and most rows are dominated by a few keys, so
    # one bf16 rounding of the weights alone exceeds 2e-3: this runs the
    # precise two-term weights, as the host drop-in does.
    d = _block(6, 4, 8192, 8192, 0, 16, 2, 512, 1e6, True, softcap=50.0, scale=1.0,
               precise=True)
    _check_rows(d, 2, 96, seed=11)
