"""Multi-GPU layout helpers for canvas attention.

Attention units (sequence, kv head) are independent (src/model/attention.rs:
116 runs them as independent tasks; GQA groups stay with their kv head,
attention.rs:149), so ranks can own disjoint units with no collective on the
attention itself. Two layouts are supported:

* batch sharding (weak scaling, what bench.py runs): rank r owns whole
  sequences; nothing is exchanged.
* head sharding: rank r owns a contiguous range of kv heads (and their query
  heads) for every sequence. The layer's o_proj (src/model/forward.rs:345)
  consumes full [tokens, n_head * head_dim] rows, so the head slices are
  reassembled with one all-gather (NCCL over NVLink on GPUs, gloo in tests).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    kv_begin: int
    kv_end: int
    q_begin: int
    q_end: int


def batch_range(batch: int, world: int, rank: int) -> range:
    """Contiguous block of sequences owned by `rank` (balanced to +-1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def head_shard(n_head: int, n_head_kv: int, world: int, rank: int) -> HeadShard:
    """kv heads [kv_begin, kv_end) and their query heads owned by `rank`.

    n_head_kv must divide evenly over the ranks so every rank holds whole GQA
    groups and the gathered output has a uniform per-rank slice.
    """
    if n_head % n_head_kv:
        raise ValueError("n_head must be a multiple of n_head_kv")
    if n_head_kv % world:
        raise ValueError(f"n_head_kv={n_head_kv} does not split over {world} ranks")
    g = n_head // n_head_kv
    per = n_head_kv // world
    kv0 = rank * per
    return HeadShard(kv0, kv0 + per, kv0 * g, (kv0 + per) * g)


def gather_heads(local_out, group=None):
    """Reassembles head-sharded outputs.

    local_out: [tokens, local_heads, head_dim] tensor of this rank (its
    contiguous query-head range). Returns [tokens, world * local_heads,
    head_dim] with rank r's heads at [r * local_heads, (r + 1) * local_heads),
    i.e. the reference's out layout [tokens, n_head * head_dim].
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    tokens, lh, hd = local_out.shape
    # One all-gather of contiguous rank slices, then a single permute into
    # head order: [world, tokens, lh, hd] -> [tokens, world, lh, hd].
    buf = torch.empty((world, tokens, lh, hd), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf.view(-1), local_out.contiguous().view(-1), group=group)
    return buf.permute(1, 0, 2, 3).reshape(tokens, world * lh, hd)


class PeerRows:
    """Receive buffers of a head-sharded layer, written directly by every rank.

    Each rank allocates one [tokens, n_head, head_dim] buffer and exports it;
    the others map it (CUDA IPC over NVLink). A rank then runs its attention
    with `out` = its own head slice of its buffer (out_row_stride = n_head *
    head_dim) and `peer_out` = the same slice of every other rank's buffer:
    the attention epilogue stores each finished tile into all of them, so
    after a barrier every rank holds the full rows o_proj consumes
    (src/model/forward.rs:345), with no all-gather and no permute afterwards.

    slice_args(shard) gives (out tensor view, peer pointers, out_row_stride)
    for that rank's head range. Peers may overwrite a buffer on the next call,
    so its owner must consume it before the ranks pass the next barrier.
    """

    def __init__(self, tokens: int, n_head: int, head_dim: int, dtype=None, group=None):
        import torch
        import torch.distributed as dist
        import canvas_attn as ca
        self._ca = ca
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        dtype = dtype or torch.bfloat16
        self.buf = torch.empty((tokens, n_head, head_dim), dtype=dtype, device="cuda")
        self.n_head, self.head_dim = n_head, head_dim
        mine = ca.ipc_export(self.buf)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        base = self.buf.data_ptr()
        self.peers = []  # (rank, mapped base address of that rank's buffer)
        for r, (h, off) in enumerate(handles):
            if r != self.rank:
                self.peers.append((r, ca.ipc_import(h, off)))
        self._base = base

    def slice_args(self, shard: HeadShard):
        """Output view and peer addresses of query heads [q_begin, q_end)."""
        esz = self.buf.element_size()
        off = shard.q_begin * self.head_dim * esz
        out = self.buf[:, shard.q_begin:shard.q_end]
        return out, [p + off for _, p in self.peers], self.n_head * self.head_dim

    def close(self):
        for _, p in self.peers:
            self._ca.ipc_close(p)
        self.peers = []
