"""The no-allocation entry point (ca_attention_block_dev_noalloc).

Some callers cannot allocate device memory: a host that links only this
library and owns no CUDA allocator, or a framework that owns every device
allocation and forbids extra cudaMalloc calls. For them the fused attention
block keeps its scratch (the normed, rotated queries) in a fixed 16 MiB array
compiled into the library. This test calls that entry point through the C ABI
twice in a row, with different inputs, and checks each result against the
regular entry point (which uses a caller-allocated scratch buffer) within the
tests' tolerance.

Which shapes pass through the scratch is observable on the regular entry
point: its caller-owned q_work is pre-filled with NaN, and the shapes whose
queries go through the scratch leave it fully written, while head_dim-128
calls that rotate Q inside the attention kernel leave it untouched. The
shapes below cover both, so a wrong or unusable scratch address would fail
the comparison. The test also checks that an oversized request that needs
the scratch is refused before anything runs, and that one that does not
need it is accepted. The file name makes pytest collect it last, and it needs
no state from other tests.
"""
import ctypes

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


# (B, n_active, n_total, H, Hkv, head_dim, queries pass through the scratch)
SHAPES = [
    (2, 300, 300, 8, 2, 64, True),      # head_dim 64: separate pre-ops pass
    (2, 32, 400, 16, 4, 128, True),     # fewer than 512 keys: separate pre-ops pass
    (4, 32, 1100, 32, 8, 128, False),   # c4-like: Q rotated inside the attention kernel
]


@pytest.mark.parametrize("B,na,n_total,H,Hkv,hd,uses_scratch", SHAPES)
def test_noalloc_matches_regular_entry_on_two_calls_in_a_row(B, na, n_total, H, Hkv, hd,
                                                              uses_scratch):
    rope = torch.from_numpy(ca.build_rope_cache(4096, hd, 5e5)).cuda()
    for call, seed in enumerate((101, 202)):
        q, k, v, ck, cv, pos, wq, wk = _inputs(seed + hd, B, na, n_total, H, Hkv, hd)
        # Regular entry point: caller-allocated scratch, its own cache copy.
        ck_ref, cv_ref = ck.clone(), cv.clone()
        out_ref = torch.empty(B, na, H, hd, device="cuda")
        q_work = torch.full((B, na, H, hd), float("nan"), dtype=torch.bfloat16, device="cuda")
        a = _args(q, k, v, ck_ref, cv_ref, pos, wq, wk, rope, out_ref, q_work, B, na, n_total,
                  H, Hkv, hd)
        assert ca.lib.ca_attention_block_dev(ctypes.byref(a), None) == ca.CA_OK
        torch.cuda.synchronize()
        written = not torch.isnan(q_work.float()).any().item()
        untouched = torch.isnan(q_work.float()).all().item()
        assert (written if uses_scratch else untouched), "unexpected pre-ops path"
        # No-allocation entry point: q_work left NULL.
        out = torch.full((B, na, H, hd), float("nan"), device="cuda")
        a = _args(q, k, v, ck, cv, pos, wq, wk, rope, out, None, B, na, n_total, H, Hkv, hd)
        assert ca.lib.ca_attention_block_dev_noalloc(ctypes.byref(a), None) == ca.CA_OK
        torch.cuda.synchronize()
        assert ca.device_status() == ca.CA_OK
        check_close(out.cpu().numpy(), out_ref.cpu().numpy(), H, hd,
                    what=f"noalloc call {call} hd={hd} keys={n_total}")
        assert torch.equal(ck, ck_ref) and torch.equal(cv, cv_ref)


def test_noalloc_rejects_requests_beyond_its_scratch():
    # head_dim 64 passes the queries through the scratch: 8 x 4096 x 16 x 64
    # bf16 = 64 MiB > 16 MiB is refused before any launch.
    B, na, H, hd = 8, 4096, 16, 64
    dummy = torch.empty(16, device="cuda")
    a = ca.make_block_args(dummy, dummy, dummy, batch=B, n_active=na, active_pos=dummy,
                           rope=dummy, rope_len=4096, rope_dim=hd, cache_k=dummy,
                           cache_v=dummy, n_total=na, q_work=None, out=dummy, n_head=H,
                           n_head_kv=H, head_dim=hd)
    assert ca.lib.ca_attention_block_dev_noalloc(ctypes.byref(a), None) == ca.CA_ERR_SCRATCH
    # Factors whose product wraps 64 bits are refused too, not wrapped past the check.
    a.batch, a.n_active, a.n_head, a.head_dim = 2 ** 30, 2 ** 30, 2 ** 30, 64
    assert ca.lib.ca_attention_block_dev_noalloc(ctypes.byref(a), None) == ca.CA_ERR_SCRATCH
    assert "scratch" in ca.status_string(ca.CA_ERR_SCRATCH)


def test_noalloc_accepts_large_calls_that_need_no_scratch():
    # 32 MiB of queries, but head_dim 128 with 1024 CTAs and 4096 keys rotates
    # Q inside the attention kernel: nothing goes through the scratch.
    B, na, n_total, H, Hkv, hd = 1, 4096, 4096, 32, 32, 128
    assert B * na * H * hd * 2 > ca.NOALLOC_SCRATCH_BYTES
    rope = torch.from_numpy(ca.build_rope_cache(4096, hd, 5e4)).cuda()
    q, k, v, ck, cv, pos, wq, wk = _inputs(7, B, na, n_total, H, Hkv, hd)
    ck_ref, cv_ref = ck.clone(), cv.clone()
    out_ref = torch.empty(B, na, H, hd, device="cuda")
    q_work = torch.empty(B, na, H, hd, dtype=torch.bfloat16, device="cuda")
    a = _args(q, k, v, ck_ref, cv_ref, pos, wq, wk, rope, out_ref, q_work, B, na, n_total, H,
              Hkv, hd)
    assert ca.lib.ca_attention_block_dev(ctypes.byref(a), None) == ca.CA_OK
    out = torch.empty(B, na, H, hd, device="cuda")
    a = _args(q, k, v, ck, cv, pos, wq, wk, rope, out, None, B, na, n_total, H, Hkv, hd)
    assert ca.lib.ca_attention_block_dev_noalloc(ctypes.byref(a), None) == ca.CA_OK
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    check_close(out.cpu().numpy(), out_ref.cpu().numpy(), H, hd, what="noalloc, no scratch")
