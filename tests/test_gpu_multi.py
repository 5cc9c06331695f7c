"""Head sharding across two GPUs (skipped with fewer than 2 GPUs).

Each rank runs the fused attention block on its own kv heads (and their
query heads) of the same seeded batch, and the head slices are reassembled
into [tokens, n_head, head_dim] rows, the layout o_proj consumes
(src/model/forward.rs:345): once with an NCCL all-gather, once by the
attention epilogue storing its tiles straight into both ranks' receive
buffers over NVLink (CUDA IPC peer mappings). A kv head's work does not
depend on the other heads, so both gathered results must equal a single-GPU
run bit for bit. NVLS is off (NCCL_NVLS_ENABLE=0) and the peer stores are
plain st.global, no multicast."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

B, S, H, HKV, HD = 2, 640, 8, 4, 128


def _inputs():
    g = torch.Generator().manual_seed(77)
    q = torch.randn(B, S, H, HD, generator=g).to(torch.bfloat16)
    k = torch.randn(B, S, HKV, HD, generator=g).to(torch.bfloat16)
    v = torch.randn(B, S, HKV, HD, generator=g).to(torch.bfloat16)
    wq = torch.rand(HD, generator=g) + 0.5
    wk = torch.rand(HD, generator=g) + 0.5
    return q, k, v, wq, wk


def _block(q, k, v, wq, wk, h, hkv, dev, out=None, peer_out=None, out_row_stride=0,
           out_multicast=None):
    import canvas_attn as ca
    rope = torch.from_numpy(ca.build_rope_cache(4096, HD, 5e4)).to(dev)
    pos = torch.arange(S, dtype=torch.int32, device=dev).repeat(B, 1).contiguous()
    cache_k = torch.zeros(B, S, hkv, HD, dtype=torch.bfloat16, device=dev)
    cache_v = torch.zeros_like(cache_k)
    q_work = torch.empty(B, S, h, HD, dtype=torch.bfloat16, device=dev)
    if out is None:
        out = torch.empty(B, S, h, HD, dtype=torch.bfloat16, device=dev)
    ca.attention_block_dev(q.contiguous().to(dev), k.contiguous().to(dev),
                           v.contiguous().to(dev), batch=B, n_active=S, active_pos=pos,
                           rope=rope, rope_len=4096, rope_dim=HD, cache_k=cache_k,
                           cache_v=cache_v, n_total=S, q_work=q_work, out=out, n_head=h,
                           n_head_kv=hkv, head_dim=HD, q_norm_w=wq.to(dev), k_norm_w=wk.to(dev),
                           rms_eps=1e-6, scale=HD ** -0.5, peer_out=peer_out,
                           out_row_stride=out_row_stride, out_multicast=out_multicast)
    return out


def _worker(rank, world, port, result_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [os.path.join(root, "diffuse-rs_b200"), root]
    import torch.distributed as dist
    import canvas_attn as ca
    from canvas_attn.sharding import PeerRows, gather_heads, head_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, k, v, wq, wk = _inputs()
        sh = head_shard(H, HKV, world, rank)
        out = _block(q[:, :, sh.q_begin:sh.q_end], k[:, :, sh.kv_begin:sh.kv_end],
                     v[:, :, sh.kv_begin:sh.kv_end], wq, wk, sh.q_end - sh.q_begin,
                     sh.kv_end - sh.kv_begin, dev)
        full = gather_heads(out.view(B * S, sh.q_end - sh.q_begin, HD))
        # Peer form: the epilogue writes both ranks' receive buffers.
        recv = PeerRows(B * S, H, HD)
        pout, peers, ors = recv.slice_args(sh)
        _block(q[:, :, sh.q_begin:sh.q_end], k[:, :, sh.kv_begin:sh.kv_end],
               v[:, :, sh.kv_begin:sh.kv_end], wq, wk, sh.q_end - sh.q_begin,
               sh.kv_end - sh.kv_begin, dev, out=pout, peer_out=peers, out_row_stride=ors)
        torch.cuda.synchronize()
        dist.barrier()
        assert ca.device_status() == ca.CA_OK
        if rank == 0:
            ref = _block(q, k, v, wq, wk, H, HKV, dev).view(B * S, H, HD)
            torch.cuda.synchronize()
            ok = torch.equal(full, ref) and torch.equal(recv.buf, ref)
            diff = max((full.float() - ref.float()).abs().max().item(),
                       (recv.buf.float() - ref.float()).abs().max().item())
            with open(result_path, "w") as f:
                f.write(f"{int(ok)} {diff}\n")
        dist.barrier()
        recv.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_head_sharded_block_gathers_match_one_gpu(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    res = tmp_path / "result.txt"
    mp.spawn(_worker, args=(2, port, str(res)), nprocs=2, join=True)
    ok, diff = res.read_text().split()
    assert ok == "1", f"gathered head-sharded output differs (max abs diff {diff})"


def _mc_worker(rank, world, port, result_path):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [os.path.join(root, "diffuse-rs_b200"), root]
    import torch.distributed as dist
    import canvas_attn as ca
    from canvas_attn.sharding import MulticastRows, head_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, k, v, wq, wk = _inputs()
        sh = head_shard(H, HKV, world, rank)
        recv = MulticastRows(B * S, H, HD)
        ok_all = [None] * world
        dist.all_gather_object(ok_all, (recv.available, recv.why))
        if not all(a for a, _ in ok_all):
            if rank == 0:
                why = next(w for a, w in ok_all if not a)
                with open(result_path, "w") as f:
                    f.write(f"skip {why}\n")
            return
        recv.buf.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        # Two calls in a row into the same buffers (the second overwrites).
        for _ in range(2):
            mout, mc, ors = recv.slice_args(sh)
            _block(q[:, :, sh.q_begin:sh.q_end], k[:, :, sh.kv_begin:sh.kv_end],
                   v[:, :, sh.kv_begin:sh.kv_end], wq, wk, sh.q_end - sh.q_begin,
                   sh.kv_end - sh.kv_begin, dev, out=mout, out_row_stride=ors,
                   out_multicast=mc)
            torch.cuda.synchronize()
            dist.barrier()
        assert ca.device_status() == ca.CA_OK
        ref = _block(q, k, v, wq, wk, H, HKV, dev).view(B * S, H, HD)
        torch.cuda.synchronize()
        ok = torch.equal(recv.buf, ref)
        diff = (recv.buf.float() - ref.float()).abs().nan_to_num(nan=1e9).max().item()
        res = [None] * world
        dist.all_gather_object(res, (ok, diff))
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(f"{int(all(o for o, _ in res))} {max(d for _, d in res)}\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_head_sharded_block_multicast_rows_match_one_gpu(tmp_path):
    """The epilogue's multimem stores through an NVLS multicast address fill
    every rank's receive buffer (each rank's buffer is checked, not only
    rank 0's) with the one-GPU rows, bit for bit."""
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    res = tmp_path / "result.txt"
    mp.spawn(_mc_worker, args=(2, port, str(res)), nprocs=2, join=True)
    txt = res.read_text().split(maxsplit=1)
    if txt[0] == "skip":
        pytest.skip(txt[1].strip())
    ok, diff = txt
    assert ok == "1", f"multicast head-sharded output differs (max abs diff {diff})"
