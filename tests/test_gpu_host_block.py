"""GPU parity of the reference-shaped entry points: the host fp32 drop-in
(`attention()`, src/model/attention.rs:106) on every golden case and on
reference-style row metadata, and the fused attention block
(src/model/forward.rs:296-343) with and without an inter-step cache."""
import os

import numpy as np
import pytest
import torch

import canvas_attn as ca
from helpers import bf16_round, check_close, oracle_attention, randn
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_cases():
    z = np.load(os.path.join(GOLD, "attention_cases.npz"))
    names = sorted({k.split("/")[0] for k in z.files})
    return {n: {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")} for n in names}


CASES = golden_cases()


def host_call(c, q, k, v):
    nq, nk, h, hkv, hd = (int(x) for x in c["dims"])
    win, cp = int(c["window"]), int(c["causal_prefix"])
    s = ca.AttnShape(nq, nk, h, hkv, hd, None if win < 0 else win, None if cp < 0 else cp,
                     float(c["scale"]), float(c["softcap"]))
    qr = ca.Rows(c["q_pos"], c.get("qseq", []), c.get("qprefix", []))
    kr = ca.Rows(c["k_pos"], c.get("kseq", []))
    out = np.zeros(nq * h * hd, np.float32)
    ca.attention(out, q, k, v, s, qr, kr)
    return out


@pytest.mark.parametrize("name", sorted(CASES))
def test_host_entry_on_golden_cases(name):
    c = CASES[name]
    nq, nk, h, hkv, hd = (int(x) for x in c["dims"])
    q, k, v = (bf16_round(torch.from_numpy(c[x])).numpy() for x in ("q", "k", "v"))
    got = host_call(c, q, k, v)
    win, cp = int(c["window"]), int(c["causal_prefix"])
    ref = orc.attention(q, k, v, nq=nq, nk=nk, n_head=h, n_head_kv=hkv, head_dim=hd,
                        q_pos=c["q_pos"], k_pos=c["k_pos"], q_seq=c.get("qseq"),
                        k_seq=c.get("kseq"), q_prefix=c.get("qprefix"),
                        sliding_window=None if win < 0 else win,
                        causal_prefix=None if cp < 0 else cp, scale=float(c["scale"]),
                        softcap=float(c["softcap"]))
    check_close(got, ref, h, hd, what=name)
    if name == "uniform_scores":  # reference known answer [2, 4] (tests.rs:104-114)
        assert abs(got[0] - 2.0) < 1e-6 and abs(got[1] - 4.0) < 1e-6


def test_host_entry_block_diagonal_seq_ids_large():
    # Three sequences concatenated with seq ids and per-sequence positions,
    # plus Gemma-style per-row causal prefixes (forward.rs:153-160).
    rng = np.random.default_rng(21)
    lens = [150, 260, 90]
    H, Hkv, hd = 4, 2, 128
    pos = np.concatenate([np.arange(n) for n in lens])
    seq = np.concatenate([np.full(n, i) for i, n in enumerate(lens)])
    canvas_start = [40, 100, 0]
    prefix = np.array([canvas_start[s] for s in seq])
    n = len(pos)
    q = bf16_round(torch.from_numpy(rng.standard_normal(n * H * hd).astype(np.float32))).numpy()
    k = bf16_round(torch.from_numpy(rng.standard_normal(n * Hkv * hd).astype(np.float32))).numpy()
    v = bf16_round(torch.from_numpy(rng.standard_normal(n * Hkv * hd).astype(np.float32))).numpy()
    s = ca.AttnShape(n, n, H, Hkv, hd, scale=hd ** -0.5)
    out = np.zeros(n * H * hd, np.float32)
    ca.attention(out, q, k, v, s, ca.Rows(pos, seq, prefix), ca.Rows(pos, seq))
    ref = orc.attention(q, k, v, nq=n, nk=n, n_head=H, n_head_kv=Hkv, head_dim=hd, q_pos=pos,
                        k_pos=pos, q_seq=seq, k_seq=seq, q_prefix=prefix, scale=hd ** -0.5)
    check_close(out, ref, H, hd, what="block-diagonal + prefix")


@pytest.mark.parametrize("masks", ["none", "seq_prefix_window", "kseq_only"])
def test_host_entry_pipelined_over_query_chunks(masks):
    # Q of 4096 rows x 8 heads x 128 fp32 = 16 MiB: the host entry point runs
    # its chunked copy-in / attention / copy-out pipeline (several launches
    # over row ranges, metadata offset per chunk); results must match the
    # one-shot semantics row for row.
    rng = np.random.default_rng(5)
    n, H, Hkv, hd = 4096, 8, 2, 128
    lens = [2500, 1596]
    pos = np.concatenate([np.arange(m) for m in lens])
    seq = np.concatenate([np.full(m, i) for i, m in enumerate(lens)])
    prefix = np.array([[300, 0][s_] for s_ in seq])
    q = bf16_round(torch.from_numpy(rng.standard_normal(n * H * hd).astype(np.float32))).numpy()
    k = bf16_round(torch.from_numpy(rng.standard_normal(n * Hkv * hd).astype(np.float32))).numpy()
    v = bf16_round(torch.from_numpy(rng.standard_normal(n * Hkv * hd).astype(np.float32))).numpy()
    kw = {}
    if masks == "none":
        qr, kr = ca.Rows(np.arange(n)), ca.Rows(np.arange(n))
        shape = ca.AttnShape(n, n, H, Hkv, hd, scale=hd ** -0.5)
    elif masks == "seq_prefix_window":
        qr, kr = ca.Rows(pos, seq, prefix), ca.Rows(pos, seq)
        shape = ca.AttnShape(n, n, H, Hkv, hd, sliding_window=700, scale=hd ** -0.5)
        kw = dict(q_pos=pos, k_pos=pos, q_seq=seq, k_seq=seq, q_prefix=prefix,
                  sliding_window=700)
    else:  # key seq ids only: queries compare as sequence 0
        qr, kr = ca.Rows(np.arange(n)), ca.Rows(np.arange(n), seq)
        shape = ca.AttnShape(n, n, H, Hkv, hd, scale=hd ** -0.5)
        kw = dict(k_seq=seq)
    out = np.full(n * H * hd, np.inf, np.float32)
    ca.attention(out, q, k, v, shape, qr, kr)
    ref = orc.attention(q, k, v, nq=n, nk=n, n_head=H, n_head_kv=Hkv, head_dim=hd,
                        scale=hd ** -0.5, kind=orc.ROW_AVX2 if orc.have_avx2()
                        else orc.ROW_SCALAR, **kw)
    check_close(out, ref, H, hd, what=f"pipelined host entry ({masks})")


def _oracle_block(q, k, v, pos, wq, wk, rope, rope_dim, h, hkv, hd, eps):
    """Reference op order (forward.rs:296-310) on fp32 copies. The attention
    operands (post-RoPE Q/K) are then rounded to bf16, as the GPU's are: the
    parity protocol is bf16 operands with fp32 accumulation."""
    q = orc.norm_heads(q, wq, eps) if wq is not None else q.copy()
    k = orc.norm_heads(k, wk, eps) if wk is not None else k.copy()
    q = orc.rotate_rows(q, rope, pos, h, hd, rope_dim)
    k = orc.rotate_rows(k, rope, pos, hkv, hd, rope_dim)
    rb = lambda x: bf16_round(torch.from_numpy(x)).numpy()  # noqa: E731
    return rb(q), rb(k), v


@pytest.mark.parametrize("qk_norm,hd,rope_dim,hkv,S", [
    (False, 128, 128, 4, 600), (True, 128, 128, 4, 600),  # Q pre-ops inside the attention
    (True, 128, 128, 2, 600),
    (True, 128, 128, 4, 300),                     # < 512 keys: separate pre-ops pass
    (True, 64, 64, 2, 300), (True, 256, 256, 2, 300),  # 256: lane-paired pre-ops
    (True, 128, 64, 4, 300),                      # partial rotation
])
def test_block_without_cache(qk_norm, hd, rope_dim, hkv, S):
    B, H, Hkv = 2, 4, hkv
    eps, theta = 1e-6, 50000.0
    g = torch.Generator().manual_seed(31)
    q = bf16_round(randn(g, B, S, H, hd))
    k = bf16_round(randn(g, B, S, Hkv, hd))
    v = bf16_round(randn(g, B, S, Hkv, hd))
    wq = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    wk = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    rope = ca.build_rope_cache(4096, rope_dim, theta)
    pos = torch.arange(S, dtype=torch.int32).repeat(B, 1)
    dev = dict(q=q.to(torch.bfloat16).cuda(), k=k.to(torch.bfloat16).cuda(),
               v=v.to(torch.bfloat16).cuda())
    cache_k = torch.zeros(B, S, Hkv, hd, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    q_work = torch.empty(B, S, H, hd, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(B, S, H, hd, device="cuda")
    rope_d = torch.from_numpy(rope).cuda()
    ca.attention_block_dev(dev["q"], dev["k"], dev["v"], batch=B, n_active=S,
                           active_pos=pos.cuda(), rope=rope_d, rope_len=4096,
                           rope_dim=rope_dim,
                           cache_k=cache_k, cache_v=cache_v, n_total=S, q_work=q_work, out=out,
                           n_head=H, n_head_kv=Hkv, head_dim=hd,
                           q_norm_w=None if wq is None else wq.cuda(),
                           k_norm_w=None if wk is None else wk.cuda(), rms_eps=eps,
                           out_f32=True, scale=hd ** -0.5, precise=True)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        qq, kk, vv = _oracle_block(q[b].numpy().reshape(-1), k[b].numpy().reshape(-1),
                                   v[b].numpy().reshape(-1), np.arange(S), None if wq is None
                                   else wq.numpy(), None if wk is None else wk.numpy(), rope,
                                   rope_dim, H, Hkv, hd, eps)
        # The stored cache holds bf16 post-RoPE K (the GPU's operand).
        kc = cache_k[b].float().cpu().numpy().reshape(-1)
        np.testing.assert_allclose(kc, kk, atol=1e-2, rtol=1e-2)
        ref = oracle_attention(qq, kk, vv, nq=S, nk=S, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5)
        check_close(got[b], ref, H, hd, what=f"block qk_norm={qk_norm} hd={hd} rope_dim={rope_dim} b={b}")


def test_block_with_cache_reuse_over_steps():
    # c4-shaped (scaled down): 32 active canvas rows in the middle of the
    # sequence attend to cached prefix/suffix K/V plus themselves; the cache is
    # reused over several steps with fresh active rows each step.
    B, n_total, na, H, Hkv, hd = 2, 600, 32, 8, 2, 128
    start = 280
    active = np.arange(start, start + na)
    cached = np.concatenate([np.arange(0, start), np.arange(start + na, n_total)])
    rope = ca.build_rope_cache(4096, hd, 5e5)
    rope_d = torch.from_numpy(rope).cuda()
    g = torch.Generator().manual_seed(41)
    cache_k = bf16_round(randn(g, B, n_total, Hkv, hd)).to(torch.bfloat16).cuda()
    cache_v = bf16_round(randn(g, B, n_total, Hkv, hd)).to(torch.bfloat16).cuda()
    pos = torch.from_numpy(np.tile(active, (B, 1)).astype(np.int32)).cuda()
    q_work = torch.empty(B, na, H, hd, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(B, na, H, hd, device="cuda")
    for step in range(3):
        before_k = cache_k.float().cpu().numpy()
        before_v = cache_v.float().cpu().numpy()
        q = bf16_round(randn(g, B, na, H, hd))
        k = bf16_round(randn(g, B, na, Hkv, hd))
        v = bf16_round(randn(g, B, na, Hkv, hd))
        ca.attention_block_dev(q.to(torch.bfloat16).cuda(), k.to(torch.bfloat16).cuda(),
                               v.to(torch.bfloat16).cuda(), batch=B, n_active=na,
                               active_pos=pos, rope=rope_d, rope_len=4096, rope_dim=hd,
                               cache_k=cache_k, cache_v=cache_v, n_total=n_total,
                               q_work=q_work, out=out, n_head=H, n_head_kv=Hkv, head_dim=hd,
                               out_f32=True, scale=hd ** -0.5, precise=True)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for b in range(B):
            qq, kk, vv = _oracle_block(q[b].numpy().reshape(-1), k[b].numpy().reshape(-1),
                                       v[b].numpy().reshape(-1), active, None, None, rope, hd,
                                       H, Hkv, hd, 1e-6)
            # Keys in the reference's order: [cached asc | active asc] (forward.rs:92-96).
            kc, vc = orc.cache_gather(before_k[b].reshape(-1), before_v[b].reshape(-1),
                                      Hkv * hd, cached)
            kf = np.concatenate([kc, kk])
            vf = np.concatenate([vc, vv])
            ref = oracle_attention(qq, kf, vf, nq=na, nk=n_total, h=H, hkv=Hkv, hd=hd,
                                   q_pos=active, k_pos=np.concatenate([cached, active]),
                                   scale=hd ** -0.5)
            check_close(got[b], ref, H, hd, what=f"cached step {step} b={b}")
        # Cached rows are untouched; active rows now hold the new post-RoPE K/V.
        after_k = cache_k.float().cpu().numpy()
        np.testing.assert_array_equal(after_k[:, cached], before_k[:, cached])


def _norm_v_heads(v, hd, eps):
    """Gemma's unweighted RMSNorm of every V head (forward.rs:304-308,
    rms_norm_noscale ops.rs:117-124), one head_dim chunk at a time."""
    v = np.array(v, np.float32).reshape(-1, hd)
    return np.concatenate([orc.rms_norm_noscale(row, eps) for row in v])


@pytest.mark.parametrize("hd,rope_dim,v_norm,qk_norm,unaligned,S", [
    (192, 192, True, True, False, 300),    # head_dim outside {64,128,256}: scalar pre-ops
    (80, 80, True, True, False, 300),      # head_dim 80 (padded to 128 in the attention tile)
    (128, 40, False, True, False, 300),    # rope_dim % 16 != 0: scalar pre-ops
    (128, 128, True, False, True, 600),    # Q/K/V 2 bytes off 16-byte alignment: scalar pre-ops
    (128, 128, True, True, False, 600),    # V norm with the Q pre-ops inside the attention kernel
    (128, 128, True, True, False, 300),    # V norm in the vectorised token kernel
    (256, 256, True, True, False, 300),    # V norm in the lane-paired head_dim-256 kernel
    (64, 32, True, True, False, 300),      # partial rotation in the head_dim-64 token kernel
    (512, 512, True, True, False, 300),    # Gemma global layer: head_dim 512
    (320, 256, False, True, False, 200),   # head_dim 320 with partial rotation
])
def test_block_pre_ops_variants(hd, rope_dim, v_norm, qk_norm, unaligned, S):
    """Every form of the pre-ops pass against the reference op order
    (forward.rs:296-310): QK-norm -> Gemma V norm -> RoPE -> cache store ->
    attention."""
    B, H, Hkv = 2, 4, 2
    eps, theta = 1e-6, 10000.0
    g = torch.Generator().manual_seed(hd * 7 + rope_dim + S)
    q = bf16_round(randn(g, B, S, H, hd))
    k = bf16_round(randn(g, B, S, Hkv, hd))
    v = bf16_round(randn(g, B, S, Hkv, hd))
    wq = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    wk = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    rope = ca.build_rope_cache(4096, rope_dim, theta)

    def dev(x):
        x = x.to(torch.bfloat16)
        if not unaligned:
            return x.cuda()
        flat = torch.empty(x.numel() + 8, dtype=torch.bfloat16, device="cuda")
        view = flat[1:1 + x.numel()].view(x.shape)  # 2 bytes past a 16-byte boundary
        view.copy_(x.cuda())
        assert view.data_ptr() % 16 == 2
        return view

    pos = torch.arange(S, dtype=torch.int32).repeat(B, 1)
    cache_k = torch.zeros(B, S, Hkv, hd, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    q_work = torch.empty(B, S, H, hd, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(B, S, H, hd, device="cuda")
    ca.attention_block_dev(dev(q), dev(k), dev(v), batch=B, n_active=S, active_pos=pos.cuda(),
                           rope=torch.from_numpy(rope).cuda(), rope_len=4096, rope_dim=rope_dim,
                           cache_k=cache_k, cache_v=cache_v, n_total=S, q_work=q_work, out=out,
                           n_head=H, n_head_kv=Hkv, head_dim=hd,
                           q_norm_w=None if wq is None else wq.cuda(),
                           k_norm_w=None if wk is None else wk.cuda(), v_norm=v_norm,
                           rms_eps=eps, out_f32=True, scale=hd ** -0.5, precise=True)
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    got = out.cpu().numpy()
    what = f"pre-ops hd={hd} rope_dim={rope_dim} v_norm={v_norm} unaligned={unaligned}"
    for b in range(B):
        qq, kk, vv = _oracle_block(q[b].numpy().reshape(-1), k[b].numpy().reshape(-1),
                                   v[b].numpy().reshape(-1), np.arange(S),
                                   None if wq is None else wq.numpy(),
                                   None if wk is None else wk.numpy(), rope, rope_dim, H, Hkv,
                                   hd, eps)
        if v_norm:
            vv = bf16_round(torch.from_numpy(_norm_v_heads(vv, hd, eps))).numpy()
        # The cache holds the bf16 post-RoPE K and the bf16 (normed) V.
        np.testing.assert_allclose(cache_k[b].float().cpu().numpy().reshape(-1), kk,
                                   atol=1e-2, rtol=1e-2, err_msg=what)
        np.testing.assert_allclose(cache_v[b].float().cpu().numpy().reshape(-1), vv,
                                   atol=1e-2, rtol=1e-2, err_msg=what)
        ref = oracle_attention(qq, kk, vv, nq=S, nk=S, h=H, hkv=Hkv, hd=hd, scale=hd ** -0.5)
        check_close(got[b], ref, H, hd, what=f"{what} b={b}")


@pytest.mark.parametrize("hd,qk_norm,v_norm,gemma", [
    (128, True, False, False),   # LLaDA-style: QK-norm, 1/sqrt(d), no prefix
    (256, True, True, True),     # Gemma-style: V norm, scale 1.0, per-sequence causal prompt
    (512, True, True, True),     # Gemma global layer heads
])
def test_block_varlen_block_diagonal_batch(hd, qk_norm, v_norm, gemma):
    """forward_batch (src/model/forward.rs:118-169) through the fused block:
    ragged sequences concatenated row-wise, each row with its own position,
    keys = its own sequence only, Gemma's causal prompt up to each sequence's
    own canvas_start. Checked against the reference's block-diagonal call
    (seq ids + per-row prefix over the concatenated rows)."""
    lens = [150, 1, 300, 77]
    starts = [40, 0, 120, 77]  # canvas_start per sequence (Gemma's causal prompt)
    B, H, Hkv = len(lens), 8, 2
    eps, theta = 1e-6, 10000.0
    scale = 1.0 if gemma else hd ** -0.5
    g = torch.Generator().manual_seed(hd + 3)
    n = sum(lens)
    q = bf16_round(randn(g, n, H, hd))
    k = bf16_round(randn(g, n, Hkv, hd))
    v = bf16_round(randn(g, n, Hkv, hd))
    wq = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    wk = torch.rand(hd, generator=g) + 0.5 if qk_norm else None
    if gemma:  # keep scale-1.0 scores moderate
        wq = wq * 0.1
    rope = ca.build_rope_cache(4096, hd, theta)
    pos = np.concatenate([np.arange(m) for m in lens])
    seq = np.concatenate([np.full(m, i) for i, m in enumerate(lens)])
    cu = torch.tensor(np.cumsum([0] + lens), dtype=torch.int32, device="cuda")
    cache_k = torch.zeros(n, Hkv, hd, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    q_work = torch.empty(n, H, hd, dtype=torch.bfloat16, device="cuda")
    out = torch.full((n, H, hd), float("inf"), device="cuda")
    prefix_d = torch.tensor(starts, dtype=torch.int32, device="cuda") if gemma else None
    ca.attention_block_dev(
        *(x.to(torch.bfloat16).cuda() for x in (q, k, v)), batch=B, n_active=0,
        active_pos=torch.from_numpy(pos.astype(np.int32)).cuda(),
        rope=torch.from_numpy(rope).cuda(), rope_len=4096, rope_dim=hd, cache_k=cache_k,
        cache_v=cache_v, n_total=0, q_work=q_work, out=out, n_head=H, n_head_kv=Hkv,
        head_dim=hd, q_norm_w=None if wq is None else wq.cuda(),
        k_norm_w=None if wk is None else wk.cuda(), v_norm=v_norm, rms_eps=eps, out_f32=True,
        scale=scale, precise=True, cu_active=cu, cu_total=cu, max_active=max(lens),
        total_active=n, total_cache=n, seq_prefix=prefix_d)
    torch.cuda.synchronize()
    assert ca.device_status() == ca.CA_OK
    qq, kk, vv = _oracle_block(q.numpy().reshape(-1), k.numpy().reshape(-1),
                               v.numpy().reshape(-1), pos, None if wq is None else wq.numpy(),
                               None if wk is None else wk.numpy(), rope, hd, H, Hkv, hd, eps)
    if v_norm:
        vv = bf16_round(torch.from_numpy(_norm_v_heads(vv, hd, eps))).numpy()
    np.testing.assert_allclose(cache_k.float().cpu().numpy().reshape(-1), kk, atol=1e-2,
                               rtol=1e-2)
    prefix = np.array([starts[s_] for s_ in seq]) if gemma else None
    ref = oracle_attention(qq, kk, vv, nq=n, nk=n, h=H, hkv=Hkv, hd=hd, q_pos=pos, k_pos=pos,
                           q_seq=seq, k_seq=seq, q_prefix=prefix, scale=scale)
    check_close(out.cpu().numpy(), ref, H, hd, what=f"varlen block hd={hd} gemma={gemma}")


@pytest.mark.parametrize("n, nk, H, Hkv", [(4096, 4096, 8, 2), (32, 4128, 32, 8)])
def test_host_entry_rounds_operands_like_the_device(n, nk, H, Hkv):
    # Raw fp32 operands (not bf16-representable): large host calls round them
    # to bf16 on host threads before copying (the pipelined form at 4096
    # queries, the one-shot form for a c4-shaped call of 32 queries over
    # 4128 keys). The rounding must be the device's round-to-nearest-even, so
    # the output equals, bit for bit, the output for the same operands
    # rounded by torch beforehand; and it matches the oracle on those.
    rng = np.random.default_rng(11)
    hd = 128
    q = (rng.standard_normal(n * H * hd) * 3).astype(np.float32)
    k = (rng.standard_normal(nk * Hkv * hd) * 3).astype(np.float32)
    v = rng.standard_normal(nk * Hkv * hd).astype(np.float32)
    rnd = lambda x: bf16_round(torch.from_numpy(x)).numpy()  # noqa: E731
    s = ca.AttnShape(n, nk, H, Hkv, hd, scale=hd ** -0.5 / 3)
    qr, kr = ca.Rows(np.arange(nk - n, nk)), ca.Rows(np.arange(nk))
    out_raw = np.full(n * H * hd, np.inf, np.float32)
    out_pre = np.full(n * H * hd, np.inf, np.float32)
    ca.attention(out_raw, q, k, v, s, qr, kr)
    ca.attention(out_pre, rnd(q), rnd(k), rnd(v), s, qr, kr)
    assert np.array_equal(out_raw, out_pre)
    ref = orc.attention(rnd(q), rnd(k), rnd(v), nq=n, nk=nk, n_head=H, n_head_kv=Hkv,
                        head_dim=hd, scale=hd ** -0.5 / 3, q_pos=np.arange(nk - n, nk),
                        k_pos=np.arange(nk),
                        kind=orc.ROW_AVX2 if orc.have_avx2() else orc.ROW_SCALAR)
    check_close(out_raw, ref, H, hd, what="host-rounded operands")
