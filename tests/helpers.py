"""Shared helpers of the GPU parity tests: seeded inputs, bf16 rounding, the
oracle call on the same bf16-rounded values, and the tolerance check.

Tolerance (bf16 operands, fp32 accumulation): per element |gpu - ref| <= 2e-3
and, per (sequence, head), ||gpu - ref||_2 / ||ref||_2 <= 1e-2.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as orc

ATOL = 2e-3
REL_L2 = 1e-2


def randn(gen: torch.Generator, *shape, scale=1.0):
    return (torch.randn(*shape, generator=gen, dtype=torch.float32) * scale)


def bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def check_close(got: np.ndarray, ref: np.ndarray, n_head: int, head_dim: int,
                atol=ATOL, rel=REL_L2, what=""):
    got = np.asarray(got, dtype=np.float32).reshape(-1, n_head, head_dim)
    ref = np.asarray(ref, dtype=np.float32).reshape(-1, n_head, head_dim)
    nan_g, nan_r = np.isnan(got), np.isnan(ref)
    assert (nan_g == nan_r).all(), f"{what}: NaN pattern differs ({nan_g.sum()} vs {nan_r.sum()})"
    g = np.where(nan_g, 0, got)
    r = np.where(nan_r, 0, ref)
    err = np.abs(g - r)
    worst = np.unravel_index(np.argmax(err), err.shape)
    assert err.max() <= atol, f"{what}: max abs err {err.max():.3e} at {worst}"
    num = np.sqrt(((g - r) ** 2).sum(axis=(0, 2)))
    den = np.sqrt((r ** 2).sum(axis=(0, 2))) + 1e-30
    assert (num / den).max() <= rel, f"{what}: rel L2 {(num / den).max():.3e}"
    return float(err.max()), float((num / den).max())


def oracle_attention(q, k, v, *, nq, nk, h, hkv, hd, **kw):
    """Oracle over float tensors/arrays (already bf16-rounded by the caller)."""
    kind = orc.ROW_AVX2 if orc.have_avx2() else orc.ROW_SCALAR
    return orc.attention(np.asarray(q, np.float32).reshape(-1), np.asarray(k, np.float32).reshape(-1),
                         np.asarray(v, np.float32).reshape(-1), nq=nq, nk=nk, n_head=h,
                         n_head_kv=hkv, head_dim=hd, kind=kind, **kw)
