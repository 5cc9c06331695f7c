"""GPU parity of the one-softmax-group attention form (two CTAs per SM).

The device entry point picks it for head_dim 128 when the grid has at least
two CTAs per SM and each CTA sees at most 2048 keys (the c2 shape: GQA 7,
1024 keys). These shapes reach it: 3 sequences x 18 query tiles x 8 kv heads
= 432 CTAs (GQA 2) or 3 x 35 x 4 = 420 (GQA 4), with every mask the kernel
distinguishes (ragged ends, window bands, causal prefixes, soft-cap) and both
output types, against the oracle at the tests' usual bar."""
import pytest
import torch

from helpers import check_close, randn
from test_gpu_parity import dev_attention, ref_batched

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,S,H,Hkv", [(3, 1100, 16, 8), (3, 1100, 16, 4), (4, 1024, 28, 4)])
@pytest.mark.parametrize("precise", [False, True])
def test_one_group_dense(B, S, H, Hkv, precise):
    g = torch.Generator().manual_seed(B * 7 + S + H + Hkv)
    hd = 128
    q, k, v = randn(g, B, S, H, hd), randn(g, B, S, Hkv, hd), randn(g, B, S, Hkv, hd)
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, precise=precise)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5)
    check_close(got.numpy(), ref, H, hd, what=f"one group {B}x{S} {H}/{Hkv}")


@pytest.mark.parametrize("kw", [
    dict(sliding_window=100),
    dict(sliding_window=700),
    dict(causal_prefix=300),
    dict(softcap=50.0),
])
def test_one_group_masks(kw):
    g = torch.Generator().manual_seed(11)
    B, S, H, Hkv, hd = 3, 1100, 16, 8, 128
    q, k, v = randn(g, B, S, H, hd), randn(g, B, S, Hkv, hd), randn(g, B, S, Hkv, hd)
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, precise=True, **kw)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, **kw)
    check_close(got.numpy(), ref, H, hd, what=f"one group {kw}")


def test_one_group_bf16_output():
    g = torch.Generator().manual_seed(12)
    B, S, H, Hkv, hd = 3, 1100, 16, 8, 128
    q, k, v = randn(g, B, S, H, hd), randn(g, B, S, Hkv, hd), randn(g, B, S, Hkv, hd)
    got = dev_attention(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5, out_f32=False)
    ref = ref_batched(q, k, v, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5)
    check_close(got.numpy(), ref, H, hd, atol=6e-3, what="one group bf16 out")


def test_one_group_block_with_fused_q_norm_and_rope():
    """The fused block at the c2 shape with QK-norm: the one-group kernel
    normalises and rotates Q in its prologue (one thread per row)."""
    from test_gpu_fullsize import _block, _oracle_seq
    d = _block(21, 4, 1024, 1024, 0, 28, 4, 128, 1e6, True)
    for b in (0, 3):
        check_close(d["out"][b].numpy(), _oracle_seq(d, b), 28, 128, what=f"block seq {b}")
