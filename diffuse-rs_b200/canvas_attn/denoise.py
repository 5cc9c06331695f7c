"""The denoising step after the forward, with the per-candidate reductions on
the GPU: Denoiser::process_logits (src/model/sampler.rs:581-593).

The logits of a step stay in HBM. One ca_candidate_stats launch computes, for
every masked position of the block, the greedy token, entropy, top1 - top2
margin and top-1 probability (collect_candidates :720-749, after
suppress_mask_token / suppress_tokens :90-113); only those four values per
candidate come back to the host, where ranking and commit run as in the
reference (update_credit :597-609, rank_candidates :613-656, commit
:658-671, tokens_to_unmask :115-132 through the C ABI in f32).

Sampling at temperature > 0 (Gumbel / nucleus, pick_token :766-806) draws
from the reference's own RNG stream and is not part of this path; neither is
Remasking::Random's shuffle with the reference's StdRng (this mirror takes a
numpy Generator for it, so its order is not the reference's).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import CaError, _ptr, _stream, lib

COSINE, LINEAR = 0, 1
ENTROPY_EXIT, LOW_CONFIDENCE, MARGIN, CONFIDENCE, ENTROPY_BOUND, RANDOM = range(6)


class CaCandArgs(ctypes.Structure):
    _fields_ = [("logits", ctypes.c_void_p), ("n_vocab", ctypes.c_int64),
                ("row_stride", ctypes.c_int64), ("rows", ctypes.c_void_p),
                ("n_cand", ctypes.c_int32), ("mask_id", ctypes.c_int32),
                ("suppress", ctypes.c_void_p), ("n_suppress", ctypes.c_int32),
                ("want_entropy", ctypes.c_int32), ("want_prob", ctypes.c_int32),
                ("token", ctypes.c_void_p), ("entropy", ctypes.c_void_p),
                ("margin", ctypes.c_void_p), ("prob", ctypes.c_void_p)]


lib.ca_candidate_stats.argtypes = [ctypes.POINTER(CaCandArgs), ctypes.c_void_p]
lib.ca_candidate_stats.restype = ctypes.c_int
lib.ca_tokens_to_unmask.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_int32]
lib.ca_tokens_to_unmask.restype = ctypes.c_int64


def tokens_to_unmask(step: int, total_steps: int, masked: int, schedule: int) -> int:
    """tokens_to_unmask (src/model/sampler.rs:115-132), f32 as the reference."""
    n = int(lib.ca_tokens_to_unmask(step, total_steps, masked, schedule))
    if n < 0:
        raise CaError(n, "ca_tokens_to_unmask")
    return n


def candidate_stats(logits, rows, token, entropy=None, margin=None, prob=None, *,
                    n_vocab: int, row_stride: int = 0, mask_id: int = -1, suppress=None,
                    want_entropy: bool = True, want_prob: bool = False, stream=None) -> None:
    """ca_candidate_stats on device tensors (see include/canvas_attn.h)."""
    n_sup = 0 if suppress is None else int(suppress.numel())
    a = CaCandArgs(_ptr(logits), int(n_vocab), int(row_stride), _ptr(rows), int(rows.numel()),
                   int(mask_id), _ptr(suppress) if n_sup else None, n_sup,
                   1 if want_entropy else 0, 1 if want_prob else 0, _ptr(token),
                   _ptr(entropy), _ptr(margin), _ptr(prob))
    rc = lib.ca_candidate_stats(ctypes.byref(a), _stream(stream))
    if rc != 0:
        raise CaError(rc, "ca_candidate_stats")


@dataclass
class Candidate:
    pos: int
    token: int
    entropy: float
    margin: float
    prob: float


@dataclass
class StepParams:
    """The Denoiser parameters this step reads (src/model.rs GenerateParams)."""
    remasking: int = LOW_CONFIDENCE
    schedule: int = COSINE
    entropy_threshold: float = 0.0
    confidence_threshold: float = 0.9
    eb_entropy_bound: float = 0.0
    credit_steps: int = 0
    suppress_ids: Sequence[int] = field(default_factory=list)


class DenoiseState:
    """The canvas of one sequence: tokens, which positions are masked, and
    the credit counters (sampler.rs:430-481)."""

    def __init__(self, seq: Sequence[int], is_masked: Sequence[bool], mask_id: int):
        self.seq = np.asarray(seq, dtype=np.int32).copy()
        self.is_masked = np.asarray(is_masked, dtype=bool).copy()
        self.n_masked = int(self.is_masked.sum())
        self.mask_id = int(mask_id)
        self.prev_pick = np.full(len(self.seq), -1, dtype=np.int64)
        self.credit = np.zeros(len(self.seq), dtype=np.int64)


def collect_candidates(state: DenoiseState, logits, n_vocab: int, rng: range, shift: int,
                       params: StepParams, stream=None):
    """collect_candidates (sampler.rs:720-749) with the row reductions on the
    GPU. `logits`: device fp32 [len(seq), n_vocab]; its suppressed entries of
    the candidate rows are set to -inf, as process_logits does."""
    import torch
    pos = [p for p in rng if state.is_masked[p]]
    if not pos:
        return []
    dev = logits.device
    rows = torch.tensor([max(p - shift, 0) for p in pos], dtype=torch.int32, device=dev)
    n = len(pos)
    tok = torch.empty(n, dtype=torch.int32, device=dev)
    vals = torch.empty((3, n), dtype=torch.float32, device=dev)
    sup = (torch.tensor(list(params.suppress_ids), dtype=torch.int32, device=dev)
           if len(params.suppress_ids) else None)
    needs_entropy = params.remasking in (ENTROPY_EXIT, LOW_CONFIDENCE, ENTROPY_BOUND)
    needs_prob = params.remasking == CONFIDENCE
    candidate_stats(logits, rows, tok, vals[0], vals[1], vals[2], n_vocab=n_vocab,
                    mask_id=state.mask_id, suppress=sup, want_entropy=needs_entropy,
                    want_prob=needs_prob, stream=stream)
    tok_h = tok.cpu().numpy()
    ent, mar, prob = vals.cpu().numpy()
    return [Candidate(p, int(tok_h[i]), float(ent[i]), float(mar[i]), float(prob[i]))
            for i, p in enumerate(pos)]


def update_credit(state: DenoiseState, cands, params: StepParams) -> None:
    """update_credit (sampler.rs:597-609)."""
    if params.credit_steps == 0:
        return
    for c in cands:
        if c.token == state.prev_pick[c.pos]:
            state.credit[c.pos] += 1
        else:
            state.credit[c.pos] = 0
            state.prev_pick[c.pos] = c.token


def rank_candidates(cands, params: StepParams, local_step: int, block_steps: int,
                    rng: Optional[np.random.Generator] = None) -> int:
    """rank_candidates (sampler.rs:613-656): orders `cands` in place (stable
    sorts, as Rust's sort_by) and returns how many to unmask."""
    n = len(cands)
    schedule_n = tokens_to_unmask(local_step, block_steps, n, params.schedule)
    r = params.remasking
    f32 = lambda x: float(np.float32(x))  # noqa: E731  (thresholds are f32 in the reference)
    if r == ENTROPY_EXIT:
        cands.sort(key=lambda c: _total_key(c.entropy))
        easy = _take_while(cands, lambda c: c.entropy < f32(params.entropy_threshold))
        return min(max(schedule_n, easy), n)
    if r == LOW_CONFIDENCE:
        cands.sort(key=lambda c: _total_key(c.entropy))
        return schedule_n
    if r == MARGIN:
        cands.sort(key=lambda c: -_total_key(c.margin))
        return schedule_n
    if r == CONFIDENCE:
        cands.sort(key=lambda c: -_total_key(c.prob))
        confident = _take_while(cands, lambda c: c.prob >= f32(params.confidence_threshold))
        return min(max(schedule_n, confident), n)
    if r == ENTROPY_BOUND:
        cands.sort(key=lambda c: _total_key(c.entropy))
        confident = _take_while(cands, lambda c: c.entropy < f32(params.eb_entropy_bound))
        return min(max(confident, 1), n)
    if r == RANDOM:
        g = rng or np.random.default_rng()
        for i in range(n - 1, 0, -1):
            j = int(g.integers(0, i + 1))
            cands[i], cands[j] = cands[j], cands[i]
        return schedule_n
    raise ValueError(f"unknown remasking {r}")


def _total_key(x: float) -> int:
    """Sort key with the order of Rust's f32::total_cmp (-0.0 < +0.0, NaNs at
    the ends by sign) on the f32 value."""
    b = int(np.array(x, dtype=np.float32).view(np.int32))
    return b ^ ((b >> 31) & 0x7FFFFFFF)


def _take_while(cands, pred) -> int:
    k = 0
    for c in cands:
        if not pred(c):
            break
        k += 1
    return k


def commit(state: DenoiseState, cands, n_unmask: int, params: StepParams) -> int:
    """commit (sampler.rs:658-671): the first n_unmask ranked candidates plus
    any credit-stable ones; returns how many were committed."""
    committed = 0
    for rank, c in enumerate(cands):
        credit_ok = params.credit_steps > 0 and state.credit[c.pos] >= params.credit_steps
        if rank < n_unmask or credit_ok:
            state.seq[c.pos] = c.token
            state.is_masked[c.pos] = False
            state.n_masked -= 1
            committed += 1
    return committed


def process_logits(state: DenoiseState, logits, n_vocab: int, rng: range, shift: int,
                   local_step: int, block_steps: int, params: StepParams,
                   stream=None, shuffle_rng=None) -> int:
    """process_logits (sampler.rs:581-593) after the forward: suppress,
    collect, credit, rank, commit. Returns the number of committed tokens."""
    cands = collect_candidates(state, logits, n_vocab, rng, shift, params, stream)
    update_credit(state, cands, params)
    n_unmask = rank_candidates(cands, params, local_step, block_steps, shuffle_rng)
    return commit(state, cands, n_unmask, params)
