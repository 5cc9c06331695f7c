"""The no-allocation entry point (ca_attention_block_dev_noalloc).

Some callers cannot allocate device memory: a host that links only this
library and owns no CUDA allocator, or a framework that owns every device
allocation and forbids extra cudaMalloc calls. For them the fused attention
block keeps its scratch (the rotated queries) in a fixed 16 MiB array
compiled into the library. This test calls that entry point through the C ABI
twice in a row, with different inputs, and checks each result against the
regular entry point (which uses a caller-allocated scratch buffer) within the
tests' tolerance; it also checks that an oversized request is refused before
anything runs. The file name makes pytest collect it last, and it needs no
state from other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import canvas_attn as ca
from helpers import check_close

pytestmark = pytest.mark.gpu


def _inputs(seed, B, na, n_total, H, Hkv, hd):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bf = torch.bfloat16

    def rnd(*s):
        return torch.randn(*s, generator=g, device="cuda").to(bf)

    q, k, v = rnd(B, na, H, hd), rnd(B, na, Hkv, hd), rnd(B, na, Hkv, hd)
    cache_k, cache_v = rnd(B, n_total, Hkv, hd), rnd(B, n_total, Hkv, hd)
    start = (n_total - na) // 2
    pos = torch.arange(start, start + na, dtype=torch.int32, device="cuda").repeat(B, 1)
    wq = torch.rand(hd, generator=g, device="cuda") + 0.5
    wk = torch.rand(hd, generator=g, device="cuda") + 0.5
    return q, k, v, cache_k, cache_v, pos.contiguous(), wq, wk


def _args(q, k, v, cache_k, cache_v, pos, wq, wk, rope, out, q_work, B, na, n_total, H, Hkv,
          hd):
    return ca.make_block_args(q, k, v, batch=B, n_active=na, active_pos=pos, rope=rope,
                              rope_len=rope.numel() // hd, rope_dim=hd, cache_k=cache_k,
                              cache_v=cache_v, n_total=n_total, q_work=q_work, out=out,
                              n_head=H, n_head_kv=Hkv, head_dim=hd, q_norm_w=wq, k_norm_w=wk,
                              rms_eps=1e-6, out_f32=True, scale=hd ** -0.5)


def test_noalloc_matches_regular_entry_on_two_calls_in_a_row():
    B, na, n_total, H, Hkv, hd = 4, 32, 1100, 32, 8, 128  # c4-like, 2 MiB of scratch
    rope = torch.from_numpy(ca.build_rope_cache(4096, hd, 5e5)).cuda()
    for call, seed in enumerate((101, 202)):
        q, k, v, ck, cv, pos, wq, wk = _inputs(seed, B, na, n_total, H, Hkv, hd)
        # Regular entry point: caller-allocated scratch, its own cache copy.
        ck_ref, cv_ref = ck.clone(), cv.clone()
        out_ref = torch.empty(B, na, H, hd, device="cuda")
        q_work = torch.empty(B, na, H, hd, dtype=torch.bfloat16, device="cuda")
        a = _args(q, k, v, ck_ref, cv_ref, pos, wq, wk, rope, out_ref, q_work, B, na, n_total,
                  H, Hkv, hd)
        assert ca.lib.ca_attention_block_dev(ctypes.byref(a), None) == ca.CA_OK
        # No-allocation entry point: q_work left NULL.
        out = torch.full((B, na, H, hd), float("nan"), device="cuda")
        a = _args(q, k, v, ck, cv, pos, wq, wk, rope, out, None, B, na, n_total, H, Hkv, hd)
        assert ca.lib.ca_attention_block_dev_noalloc(ctypes.byref(a), None) == ca.CA_OK
        torch.cuda.synchronize()
        assert ca.device_status() == ca.CA_OK
        check_close(out.cpu().numpy(), out_ref.cpu().numpy(), H, hd,
                    what=f"noalloc call {call}")
        assert torch.equal(ck, ck_ref) and torch.equal(cv, cv_ref)


def test_noalloc_rejects_requests_beyond_its_scratch():
    B, na, H, hd = 8, 4096, 16, 128  # 128 MiB of rotated queries > 16 MiB
    dummy = torch.empty(16, device="cuda")
    a = ca.make_block_args(dummy, dummy, dummy, batch=B, n_active=na, active_pos=dummy,
                           rope=dummy, rope_len=4096, rope_dim=hd, cache_k=dummy,
                           cache_v=dummy, n_total=na, q_work=None, out=dummy, n_head=H,
                           n_head_kv=H, head_dim=hd)
    assert ca.lib.ca_attention_block_dev_noalloc(ctypes.byref(a), None) == ca.CA_ERR_SCRATCH
    assert "scratch" in ca.status_string(ca.CA_ERR_SCRATCH)
