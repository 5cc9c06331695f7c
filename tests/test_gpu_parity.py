"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle on the
same seeded, bf16-rounded inputs. Small and ragged shapes first, then masks.

Rows that see only a handful of keys (tiny windows, early causal-prompt rows,
very peaked soft-capped scores) are where one bf16 rounding of the softmax
weights alone reaches ~4e-3; those cases run the `precise` form (weights as
bf16 hi + lo terms), which is what the host drop-in entry point always uses.
Dense cases run the default single-term form."""
import numpy as np
import pytest
import torch

import canvas_attn as ca
from helpers import bf16_round, check_close, oracle_attention, randn
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def dev_attention(q, k, v, *, h, hkv, hd, out_f32=True, **kw):
    """q [B, Sq, H, hd], k/v [B, Sk, Hkv, hd] fp32 CPU tensors -> fp32 CPU output."""
    B, Sq = q.shape[0], q.shape[1]
    Sk = k.shape[1]
    qd = q.to(torch.bfloat16).cuda().contiguous()
    kd = k.to(torch.bfloat16).cuda().contiguous()
    vd = v.to(torch.bfloat16).cuda().contiguous()
    out = torch.full((B, Sq, h, hd), float("inf"),
                     dtype=torch.float32 if out_f32 else torch.bfloat16, device="cuda")
    ca.attention_dev(qd, kd, vd, out, batch=B, sq=Sq, sk=Sk, n_head=h, n_head_kv=hkv,
                     head_dim=hd, out_f32=out_f32, **kw)
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    return out.float().cpu()


def ref_batched(q, k, v, *, h, hkv, hd, scale, **kw):
    """Oracle per sequence of a uniform batch (the reference's block-diagonal
    batching is equivalent to separate calls, src/model/tests.rs:70-102)."""
    outs = []
    for b in range(q.shape[0]):
        outs.append(oracle_attention(bf16_round(q[b]), bf16_round(k[b]), bf16_round(v[b]),
                                     nq=q.shape[1], nk=k.shape[1], h=h, hkv=hkv, hd=hd,
                                     scale=scale, **kw))
    return np.stack(outs)


@pytest.mark.parametrize("B,Sq,Sk,H,Hkv,hd", [
    (1, 128, 128, 1, 1, 128),   # one tile
    (1, 128, 256, 2, 1, 128),   # two key tiles, GQA 2
    (2, 200, 333, 4, 4, 128),   # ragged query and key tiles
    (1, 128, 128, 32, 32, 128),  # c1 shape
    (2, 300, 300, 28, 4, 128),  # c2 GQA group 7 (126-row tiles), ragged
    (1, 77, 500, 8, 2, 64),
    (1, 130, 257, 4, 2, 256),
    (1, 64, 200, 2, 2, 192),
    (1, 100, 150, 2, 1, 72),    # head_dim padded to 128 by the TMA zero fill
    (1, 40, 4128, 32, 8, 128),  # c4-like: 32 queries x 4 heads per tile
    # Wide heads (DiffusionGemma global layers: head_dim 512, 16/2 heads):
    # two CTAs per Q tile, each owning half of O's columns.
    (1, 130, 300, 16, 2, 512),
    (2, 100, 257, 4, 1, 320),   # head_dim 320 runs the 384-column tile
    (1, 64, 129, 2, 2, 264),    # 264: the second CTA's columns are mostly padding
    (1, 33, 520, 8, 2, 384),
])
@pytest.mark.parametrize("precise", [False, True])
def test_dense_matches_oracle(B, Sq, Sk, H, Hkv, hd, precise):
    g = torch.Generator().manual_seed(B * 1000 + Sq + Sk + H + hd)
    q = randn(g, B, Sq, H, hd)
    k = randn(g, B, Sk, Hkv, hd)
    v = randn(g, B, Sk, Hkv, hd)
    scale = hd ** -0.5
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=scale, precise=precise)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=scale)
    e, r = check_close(got.numpy(), ref, H, hd, what=f"{B}x{Sq}x{Sk} {H}/{Hkv} hd{hd}")
    if precise:  # two-term weights: far inside the bound
        assert e < 5e-4, e


def test_bf16_output_matches_oracle():
    g = torch.Generator().manual_seed(5)
    q, k, v = randn(g, 2, 256, 4, 128), randn(g, 2, 256, 2, 128), randn(g, 2, 256, 2, 128)
    got = dev_attention(q, k, v, h=4, hkv=2, hd=128, scale=128 ** -0.5, out_f32=False)
    ref = ref_batched(q, k, v, h=4, hkv=2, hd=128, scale=128 ** -0.5)
    check_close(got.numpy(), ref, 4, 128, atol=6e-3, what="bf16 out")


@pytest.mark.parametrize("window", [1, 7, 100, 512])
def test_sliding_window(window):
    g = torch.Generator().manual_seed(window)
    S, H, Hkv, hd = 700, 4, 2, 128
    q, k, v = randn(g, 1, S, H, hd), randn(g, 1, S, Hkv, hd), randn(g, 1, S, Hkv, hd)
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, sliding_window=window,
                        precise=True)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, sliding_window=window)
    check_close(got.numpy(), ref, H, hd, what=f"window {window}")


def test_window_zero_gives_nan_like_reference():
    g = torch.Generator().manual_seed(9)
    q, k, v = randn(g, 1, 50, 2, 64), randn(g, 1, 60, 2, 64), randn(g, 1, 60, 2, 64)
    got = dev_attention(q, k, v, h=2, hkv=2, hd=64, scale=0.125, sliding_window=0)
    assert torch.isnan(got).all()


@pytest.mark.parametrize("prefix", [0, 37, 129, 400])
def test_causal_prefix(prefix):
    g = torch.Generator().manual_seed(prefix + 3)
    S, H, hd = 300, 2, 128
    q, k, v = randn(g, 1, S, H, hd), randn(g, 1, S, H, hd), randn(g, 1, S, H, hd)
    got = dev_attention(q, k, v, h=H, hkv=H, hd=hd, scale=hd ** -0.5, causal_prefix=prefix,
                        precise=True)
    ref = ref_batched(q, k, v, h=H, hkv=H, hd=hd, scale=hd ** -0.5, causal_prefix=prefix)
    check_close(got.numpy(), ref, H, hd, what=f"prefix {prefix}")


@pytest.mark.parametrize("softcap,scale", [(50.0, 1 / 16), (5.0, 1.0), (50.0, 1.0)])
def test_softcap_extension(softcap, scale):
    g = torch.Generator().manual_seed(int(softcap))
    S, H, Hkv, hd = 400, 4, 2, 256
    q, k, v = randn(g, 1, S, H, hd), randn(g, 1, S, Hkv, hd), randn(g, 1, S, Hkv, hd)
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=scale, softcap=softcap,
                        precise=True)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=scale, softcap=softcap)
    check_close(got.numpy(), ref, H, hd, what=f"softcap {softcap} scale {scale}")


def test_negative_scale():
    g = torch.Generator().manual_seed(77)
    q, k, v = randn(g, 1, 150, 2, 128), randn(g, 1, 150, 2, 128), randn(g, 1, 150, 2, 128)
    got = dev_attention(q, k, v, h=2, hkv=2, hd=128, scale=-0.1, precise=True)
    ref = ref_batched(q, k, v, h=2, hkv=2, hd=128, scale=-0.1)
    check_close(got.numpy(), ref, 2, 128, what="negative scale")


def test_varlen_batch():
    g = torch.Generator().manual_seed(11)
    lens_q, lens_k = [5, 300, 128, 0, 77], [40, 250, 128, 10, 77]
    H, Hkv, hd = 6, 2, 128
    tq, tk = sum(lens_q), sum(lens_k)
    q, k, v = randn(g, tq, H, hd), randn(g, tk, Hkv, hd), randn(g, tk, Hkv, hd)
    cu_q = torch.tensor(np.cumsum([0] + lens_q), dtype=torch.int32, device="cuda")
    cu_k = torch.tensor(np.cumsum([0] + lens_k), dtype=torch.int32, device="cuda")
    qd, kd, vd = (x.to(torch.bfloat16).cuda() for x in (q, k, v))
    out = torch.zeros(tq, H, hd, device="cuda")
    ca.attention_dev(qd, kd, vd, out, batch=len(lens_q), sq=0, sk=0, cu_q=cu_q, cu_k=cu_k,
                     max_sq=max(lens_q), total_q=tq, total_k=tk, n_head=H, n_head_kv=Hkv,
                     head_dim=hd, out_f32=True, scale=hd ** -0.5)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    oq = ok = 0
    for lq, lk in zip(lens_q, lens_k):
        if lq:
            ref = oracle_attention(bf16_round(q[oq:oq + lq]), bf16_round(k[ok:ok + lk]),
                                   bf16_round(v[ok:ok + lk]), nq=lq, nk=lk, h=H, hkv=Hkv, hd=hd,
                                   scale=hd ** -0.5)
            check_close(got[oq:oq + lq], ref, H, hd, what=f"varlen {lq}x{lk}")
        oq += lq
        ok += lk


@pytest.mark.parametrize("hd", [320, 512])
def test_wide_heads_with_masks_bf16_out_and_varlen(hd):
    # Gemma global-layer form: scale 1.0 and soft-cap; plus a sliding window,
    # a causal prefix, bf16 output and a varlen batch at head_dim > 256.
    g = torch.Generator().manual_seed(hd)
    S, H, Hkv = 300, 8, 1
    q, k, v = randn(g, 1, S, H, hd, scale=0.05), randn(g, 1, S, Hkv, hd), randn(g, 1, S, Hkv, hd)
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=1.0, softcap=50.0, precise=True)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=1.0, softcap=50.0)
    check_close(got.numpy(), ref, H, hd, what=f"hd {hd} soft-cap")
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, sliding_window=40,
                        causal_prefix=100, precise=True)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, sliding_window=40,
                      causal_prefix=100)
    check_close(got.numpy(), ref, H, hd, what=f"hd {hd} window + prefix")
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, out_f32=False)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5)
    check_close(got.numpy(), ref, H, hd, atol=6e-3, what=f"hd {hd} bf16 out")
    lens_q, lens_k = [70, 0, 130], [90, 20, 130]
    tq, tk = sum(lens_q), sum(lens_k)
    q, k, v = randn(g, tq, H, hd), randn(g, tk, Hkv, hd), randn(g, tk, Hkv, hd)
    cu_q = torch.tensor(np.cumsum([0] + lens_q), dtype=torch.int32, device="cuda")
    cu_k = torch.tensor(np.cumsum([0] + lens_k), dtype=torch.int32, device="cuda")
    out = torch.zeros(tq, H, hd, device="cuda")
    ca.attention_dev(*(x.to(torch.bfloat16).cuda() for x in (q, k, v)), out,
                     batch=len(lens_q), sq=0, sk=0, cu_q=cu_q, cu_k=cu_k, max_sq=max(lens_q),
                     total_q=tq, total_k=tk, n_head=H, n_head_kv=Hkv, head_dim=hd,
                     out_f32=True, scale=hd ** -0.5, precise=True)
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    got = out.cpu().numpy()
    oq = ok = 0
    for lq, lk in zip(lens_q, lens_k):
        if lq:
            ref = oracle_attention(bf16_round(q[oq:oq + lq]), bf16_round(k[ok:ok + lk]),
                                   bf16_round(v[ok:ok + lk]), nq=lq, nk=lk, h=H, hkv=Hkv,
                                   hd=hd, scale=hd ** -0.5)
            check_close(got[oq:oq + lq], ref, H, hd, what=f"hd {hd} varlen {lq}x{lk}")
        oq += lq
        ok += lk


def test_head_dim_beyond_512_is_unsupported():
    x = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ca.CaError) as e:
        ca.attention_dev(x, x, x, x, batch=1, sq=1, sk=1, n_head=1, n_head_kv=1, head_dim=520)
    assert e.value.status == ca.CA_ERR_UNSUPPORTED
