"""GPU parity of the staged-ring pre-ops pass (full rotation at head_dim 64,
128 and 256, passes of at least 256K rows): the normed and rotated Q in
q_work and the post-RoPE K / (Gemma-normed) V in the cache against the
oracle's restatement of the reference op order (norm_heads, rotate_rows,
rms_norm_noscale; src/model/forward.rs:296-320), bit for bit, plus sampled
attention rows of the same call.

Token counts are not multiples of the ring's tokens per stage, so the last
stage is partial; one case is a variable-length batch (cache rows at
cu_total[b] + position)."""
import numpy as np
import pytest
import torch

import canvas_attn as ca
from helpers import bf16_round, check_close, randn
from oracle import oracle as orc
from test_gpu_host_block import _norm_v_heads, _oracle_block

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hd,B,na,H,Hkv,qk_norm,v_norm,varlen", [
    (128, 4, 4099, 16, 8, True, False, False),   # c3-like rows; Q in the pass (grid > 8 waves)
    (128, 4, 4099, 16, 8, False, True, False),   # no QK-norm, Gemma V norm
    (256, 2, 4099, 16, 8, True, True, False),    # c5-like rows
    (64, 2, 4099, 32, 16, True, False, False),
    (128, 4, 4099, 16, 8, True, True, True),     # variable-length batch
])
def test_ring_pre_ops_match_oracle(hd, B, na, H, Hkv, qk_norm, v_norm, varlen):
    eps, theta = 1e-6, 1e6
    g = torch.Generator().manual_seed(hd + na + H + int(varlen))
    q = bf16_round(randn(g, B, na, H, hd))
    k = bf16_round(randn(g, B, na, Hkv, hd))
    v = bf16_round(randn(g, B, na, Hkv, hd))
    wq = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    wk = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    rope_len = 8192
    rope = ca.build_rope_cache(rope_len, hd, theta)
    rope_d = torch.from_numpy(rope).cuda()
    pos = np.arange(na)
    common = dict(rope=rope_d, rope_len=rope_len, rope_dim=hd, n_head=H, n_head_kv=Hkv,
                  head_dim=hd, q_norm_w=None if wq is None else wq.cuda(),
                  k_norm_w=None if wk is None else wk.cuda(), v_norm=v_norm, rms_eps=eps,
                  out_f32=True, scale=hd ** -0.5, precise=True)
    if varlen:
        n = B * na
        cu = torch.tensor([b * na for b in range(B + 1)], dtype=torch.int32, device="cuda")
        cache_k = torch.zeros(n, Hkv, hd, dtype=torch.bfloat16, device="cuda")
        cache_v = torch.zeros_like(cache_k)
        q_work = torch.empty(n, H, hd, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(n, H, hd, device="cuda")
        ca.attention_block_dev(
            *(x.reshape(n, -1, hd).to(torch.bfloat16).cuda() for x in (q, k, v)), batch=B,
            n_active=0, active_pos=torch.from_numpy(np.tile(pos, B).astype(np.int32)).cuda(),
            cache_k=cache_k, cache_v=cache_v, n_total=0, q_work=q_work, out=out,
            cu_active=cu, cu_total=cu, max_active=na, total_active=n, total_cache=n, **common)
        cache_k, cache_v = cache_k.view(B, na, Hkv, hd), cache_v.view(B, na, Hkv, hd)
        q_work, out = q_work.view(B, na, H, hd), out.view(B, na, H, hd)
    else:
        cache_k = torch.zeros(B, na, Hkv, hd, dtype=torch.bfloat16, device="cuda")
        cache_v = torch.zeros_like(cache_k)
        q_work = torch.empty(B, na, H, hd, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(B, na, H, hd, device="cuda")
        ca.attention_block_dev(
            *(x.to(torch.bfloat16).cuda() for x in (q, k, v)), batch=B, n_active=na,
            active_pos=torch.from_numpy(pos.astype(np.int32)).repeat(B, 1).cuda(),
            cache_k=cache_k, cache_v=cache_v, n_total=na, q_work=q_work, out=out, **common)
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    what = f"ring pre-ops hd={hd} qk_norm={qk_norm} v_norm={v_norm} varlen={varlen}"
    for b in (0, B - 1):
        qq, kk, vv = _oracle_block(q[b].numpy().reshape(-1), k[b].numpy().reshape(-1),
                                   v[b].numpy().reshape(-1), pos,
                                   None if wq is None else wq.numpy(),
                                   None if wk is None else wk.numpy(), rope, hd, H, Hkv, hd, eps)
        if v_norm:
            vv = _norm_v_heads(vv, hd, eps)
        vv = bf16_round(torch.from_numpy(np.asarray(vv, np.float32))).numpy()
        # Same arithmetic in the same order: bit-identical bf16 results.
        np.testing.assert_array_equal(q_work[b].float().cpu().numpy().reshape(-1), qq,
                                      err_msg=f"{what} q b={b}")
        np.testing.assert_array_equal(cache_k[b].float().cpu().numpy().reshape(-1), kk,
                                      err_msg=f"{what} k b={b}")
        np.testing.assert_array_equal(cache_v[b].float().cpu().numpy().reshape(-1), vv,
                                      err_msg=f"{what} v b={b}")
        # A seeded sample of attention rows of this sequence.
        rng = np.random.default_rng(b)
        tasks = np.sort(rng.choice(H * na, size=64, replace=False)).astype(np.int64)
        ref = orc.attention(qq, kk, vv, nq=na, nk=na, n_head=H, n_head_kv=Hkv, head_dim=hd,
                            scale=hd ** -0.5, tasks=tasks,
                            kind=orc.ROW_AVX2 if orc.have_avx2() else orc.ROW_SCALAR)
        ref = ref.reshape(na, H, hd)
        heads, rows = tasks // na, tasks % na
        got = out[b].cpu().numpy()[rows, heads]
        check_close(got.reshape(-1, 1, hd), ref[rows, heads].reshape(-1, 1, hd), 1, hd,
                    what=f"{what} attention b={b}")
