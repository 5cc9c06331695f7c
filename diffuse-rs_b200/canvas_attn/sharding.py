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


class MulticastRows:
    """Receive buffers of a head-sharded layer written through NVLink multicast.

    Each rank allocates its [tokens, n_head, head_dim] buffer from torch's
    symmetric memory, which binds the same-offset buffers of every rank to
    one NVLS multicast object (plumbing only: the writes are the attention
    epilogue's own multimem stores). A rank runs its attention with `out` =
    its head slice of its buffer and `out_multicast` = the multicast address
    of that slice: every output row crosses this GPU's NVLink once and the
    switch writes it into every rank's buffer, where PeerRows sends it once
    per peer. After a barrier every rank holds the full rows o_proj consumes
    (src/model/forward.rs:345).

    `available` is False (and `why` says why) when the box, driver or torch
    build offers no multicast; callers then fall back to PeerRows or NCCL.
    """

    def __init__(self, tokens: int, n_head: int, head_dim: int, dtype=None, group=None):
        import torch
        import torch.distributed as dist
        self.n_head, self.head_dim = n_head, head_dim
        self.rank = dist.get_rank(group)
        self.available, self.why, self.mc = False, "", 0
        dtype = dtype or torch.bfloat16
        try:
            import torch.distributed._symmetric_memory as symm_mem
            grp = group if group is not None else dist.group.WORLD
            name = grp.group_name
            self.buf = symm_mem.empty((tokens, n_head, head_dim), dtype=dtype,
                                      device=torch.device("cuda", torch.cuda.current_device()))
            self.handle = symm_mem.rendezvous(self.buf, name)
            mc = int(self.handle.multicast_ptr or 0)  # 0: no multicast object
            base = int(self.handle.buffer_ptrs[self.rank])
            off = self.buf.data_ptr() - base
            nbytes = self.buf.numel() * self.buf.element_size()
            if mc == 0:
                self.why = "no NVLS multicast support on this box"
            elif off < 0 or off + nbytes > int(self.handle.buffer_size) or mc % 16 or off % 16:
                self.why = "buffer outside its symmetric allocation"
            else:
                self.mc = mc + off
                self.available = True
        except Exception as e:  # noqa: BLE001 - reported, never fatal
            self.why = f"symmetric memory unavailable: {type(e).__name__}: {e}"
        if not self.available and not hasattr(self, "buf"):
            self.buf = torch.empty((tokens, n_head, head_dim), dtype=dtype, device="cuda")

    def barrier(self, stream=None):
        """Stream-ordered barrier over the group through the symmetric
        allocation's signal pads (a small kernel on `stream`, after the
        layer's kernels): once it completes on a rank, every rank's stores
        issued before its own barrier are in place. Measured on B200 at two
        ranks: 12 us, against 22 us for a 4-byte NCCL all_reduce."""
        import torch
        with torch.cuda.stream(stream or torch.cuda.current_stream()):
            self.handle.barrier(channel=0)

    def slice_args(self, shard: HeadShard):
        """Output view, multicast address and out_row_stride of query heads
        [q_begin, q_end)."""
        esz = self.buf.element_size()
        off = shard.q_begin * self.head_dim * esz
        out = self.buf[:, shard.q_begin:shard.q_end]
        return out, self.mc + off, self.n_head * self.head_dim


# ---------------------------------------------------------------- failures
# Host-side failure detection for multi-rank layers. The reference has no
# multi-process path (its failure handling is request-level); these helpers
# make a bad or missing rank surface as an error on every rank before any
# kernel or collective of the next step is launched, instead of a hang.


class ShardMismatch(ValueError):
    """The ranks disagree on a layer's shape or sharding arguments."""


class RankFailed(RuntimeError):
    """Another rank reported a failure (between steps)."""

    def __init__(self, rank: int, what: str):
        super().__init__(f"rank {rank} failed: {what}")
        self.rank = rank
        self.what = what


def agree_on_layer(fields: dict, group=None) -> None:
    """Checks that every rank passes the same layer arguments.

    fields: plain values (ints, floats, strings) describing the call, e.g.
    tokens, n_head, n_head_kv, head_dim, world. Exchanged with one
    all_gather_object; on any difference every rank raises ShardMismatch
    naming the first differing field and the ranks' values, so no rank goes
    on to launch a layer whose peers would wait for it forever.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    mine = tuple(sorted(fields.items()))
    every = [None] * world
    dist.all_gather_object(every, mine, group=group)
    for r, other in enumerate(every):
        if other != mine:
            a, b = dict(mine), dict(other)
            diff = sorted(k for k in set(a) | set(b) if a.get(k) != b.get(k))
            k = diff[0] if diff else "?"
            raise ShardMismatch(f"layer arguments differ: {k} = {a.get(k)!r} here, "
                                f"{b.get(k)!r} on rank {r}")


class FailureBoard:
    """Failure notices between steps, on the process group's key-value store.

    A rank that fails inside `step()` writes `<prefix>/<rank>` before the
    exception leaves it; every rank calls `check()` before launching the next
    step and raises RankFailed for the first failed rank it finds. A rank
    therefore leaves only between steps, with none of its work in flight, and
    the others learn of it on the host. `wait_for(rank, seconds)` polls until
    a given rank has reported (tests and drivers that expect a failure).
    """

    def __init__(self, prefix: str = "ca_fail", store=None, group=None):
        import torch.distributed as dist
        from torch.distributed import distributed_c10d as c10d

        self.store = store if store is not None else c10d._get_default_store()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.prefix = prefix

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def report(self, exc: BaseException) -> None:
        self.store.set(self._key(self.rank), f"{type(exc).__name__}: {exc}")

    def check(self) -> None:
        for r in range(self.world):
            if r != self.rank and self.store.check([self._key(r)]):
                raise RankFailed(r, self.store.get(self._key(r)).decode())

    def wait_for(self, rank: int, seconds: float) -> None:
        import time

        deadline = time.monotonic() + seconds
        while time.monotonic() < deadline:
            self.check()
            time.sleep(0.01)
        raise TimeoutError(f"rank {rank} reported nothing within {seconds} s")

    class _Step:
        def __init__(self, board):
            self.board = board

        def __enter__(self):
            self.board.check()
            return self

        def __exit__(self, et, ev, tb):
            if ev is not None and not isinstance(ev, RankFailed):
                self.board.report(ev)
            return False

    def step(self):
        """Context manager for one step: checks the board on entry and
        reports this rank's exception (and re-raises it) on the way out."""
        return FailureBoard._Step(self)


def init_group(backend: str, rank: int, world: int, timeout_s: float = 60.0) -> None:
    """init_process_group with a bounded rendezvous and collective timeout:
    a rank that never joins makes the others' init raise after `timeout_s`
    instead of waiting forever (and, with NCCL, a collective that does not
    complete within it is aborted by the process group's watchdog)."""
    import datetime

    import torch.distributed as dist

    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
