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


# ------------------------------------------------ host-side failure detection
def _failure_worker(rank, world, port, case, result):
    import sys
    import time
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "diffuse-rs_b200")]
    from canvas_attn.sharding import (FailureBoard, RankFailed, ShardMismatch,
                                      agree_on_layer, init_group)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if case == "never_joins":
        if rank == 1:
            result[rank] = "stayed away"
            return
        t0 = time.monotonic()
        try:
            init_group("gloo", rank, world, timeout_s=3.0)
            result[rank] = "joined"
        except Exception as e:  # rendezvous timeout
            result[rank] = f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"
        return
    init_group("gloo", rank, world, timeout_s=30.0)
    try:
        if case == "bad_shape":
            try:
                agree_on_layer(dict(tokens=4096, n_head=16, n_head_kv=16,
                                    head_dim=128 if rank == 0 else 64, world=world))
                result[rank] = "agreed"
            except ShardMismatch as e:
                result[rank] = f"mismatch: {e}"
        elif case == "rank_raises":
            board = FailureBoard()
            if rank == 1:
                try:
                    with board.step():
                        raise RuntimeError("injected failure in step 0")
                except RuntimeError:
                    result[rank] = "raised"
            else:
                try:
                    board.wait_for(1, 20.0)
                    result[rank] = "no notice"
                except RankFailed as e:
                    result[rank] = f"saw rank {e.rank}: {e.what}"
    finally:
        dist.destroy_process_group()


def _run_failure_case(case):
    world = 2
    mgr = mp.Manager()
    result = mgr.dict()
    mp.spawn(_failure_worker, args=(world, _free_port(), case, result), nprocs=world, join=True)
    return dict(result)


def test_bad_shape_on_one_rank_is_an_error_on_every_rank():
    res = _run_failure_case("bad_shape")
    assert res[0].startswith("mismatch: layer arguments differ: head_dim = 128 here, 64 on rank 1")
    assert res[1].startswith("mismatch: layer arguments differ: head_dim = 64 here, 128 on rank 0")


def test_rank_that_raises_between_steps_is_seen_by_the_others():
    res = _run_failure_case("rank_raises")
    assert res[1] == "raised"
    assert res[0] == "saw rank 1: RuntimeError: injected failure in step 0"


def test_rank_that_never_joins_times_out_the_rendezvous():
    res = _run_failure_case("never_joins")
    assert res[1] == "stayed away"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 30.0
