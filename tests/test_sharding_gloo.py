"""Multi-rank host logic on CPU (gloo, world size 2): kv-head sharding of an
attention layer and the all-gather that reassembles head outputs, checked
against the unsharded oracle; plus the batch split used by the weak-scaling
bench. The per-rank attention is computed by the oracle here (CPU test of the
layout logic; the CUDA kernel's parity is covered by the gpu tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from canvas_attn.sharding import batch_range, gather_heads, head_shard


def test_batch_range_covers_everything_once():
    for batch in (1, 7, 8, 16):
        for world in (1, 2, 4, 8):
            got = [i for r in range(world) for i in batch_range(batch, world, r)]
            assert got == list(range(batch))


def test_head_shard_keeps_gqa_groups():
    s = [head_shard(28, 4, 2, r) for r in range(2)]
    assert (s[0].q_begin, s[0].q_end, s[1].q_begin, s[1].q_end) == (0, 14, 14, 28)
    with pytest.raises(ValueError):
        head_shard(28, 4, 8, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "diffuse-rs_b200")]
    from oracle import oracle as orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nq, nk, H, Hkv, hd = 40, 60, 8, 4, 16
        rng = np.random.default_rng(0)  # same inputs on every rank
        q = rng.standard_normal((nq, H, hd), dtype=np.float32)
        k = rng.standard_normal((nk, Hkv, hd), dtype=np.float32)
        v = rng.standard_normal((nk, Hkv, hd), dtype=np.float32)
        sh = head_shard(H, Hkv, world, rank)
        ql = np.ascontiguousarray(q[:, sh.q_begin:sh.q_end])
        kl = np.ascontiguousarray(k[:, sh.kv_begin:sh.kv_end])
        vl = np.ascontiguousarray(v[:, sh.kv_begin:sh.kv_end])
        local = orc.attention(ql, kl, vl, nq=nq, nk=nk, n_head=sh.q_end - sh.q_begin,
                              n_head_kv=sh.kv_end - sh.kv_begin, head_dim=hd, scale=0.25,
                              sliding_window=9)
        full = gather_heads(torch.from_numpy(local.reshape(nq, -1, hd)))
        ref = orc.attention(q, k, v, nq=nq, nk=nk, n_head=H, n_head_kv=Hkv, head_dim=hd,
                            scale=0.25, sliding_window=9)
        result[rank] = float(np.abs(full.numpy().reshape(-1) - ref).max())
    finally:
        dist.destroy_process_group()


def test_head_sharded_layer_gathers_to_unsharded_result():
    world = 2
    mgr = mp.Manager()
    result = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), result), nprocs=world, join=True)
    assert len(result) == world
    for r in range(world):
        assert result[r] == 0.0, result[r]  # same rows, same order: bit-exact
