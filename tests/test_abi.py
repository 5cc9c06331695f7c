"""The C-ABI library loads, exports every symbol include/canvas_attn.h
declares, and validates arguments -- all without a GPU (no compute calls)."""
import ctypes
import os
import re

import numpy as np

import canvas_attn as ca
from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "canvas_attn.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ca_[a-z0-9_]+)\s*\(", src)))


def test_header_and_mirror_agree():
    assert declared_symbols() == sorted(ca.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(ca.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_version_and_status_strings():
    assert "sm_100a" in ca.version()
    assert ca.status_string(ca.CA_OK) == "ok"
    assert "timed out" in ca.status_string(ca.CA_ERR_TIMEOUT)


def test_rope_table_matches_oracle_bit_exact():
    # build_rope_cache_ff (src/model/ops.rs:398-416): same f32 formula.
    for theta, dim in ((500000.0, 128), (1e6, 128), (10000.0, 256), (50000.0, 64)):
        a = ca.build_rope_cache(300, dim, theta)
        b = orc.build_rope_cache(300, dim, theta)
        np.testing.assert_array_equal(a, b)
    ff = np.linspace(1.0, 4.0, 32).astype(np.float32)
    np.testing.assert_array_equal(ca.build_rope_cache(50, 64, 1e4, ff),
                                  orc.build_rope_cache(50, 64, 1e4, ff))


def test_dev_entry_rejects_bad_arguments_without_touching_the_gpu():
    a = ca.make_dev_args(None, None, None, None, batch=1, sq=1, sk=1, n_head=1, n_head_kv=1,
                         head_dim=128)
    assert ca.lib.ca_attention_dev(ctypes.byref(a), None) == ca.CA_ERR_INVALID
    # Unsupported head_dim / GQA ratio / misaligned pointers are rejected up front.
    fake = 1 << 40
    a = ca.make_dev_args(fake, fake, fake, fake, batch=1, sq=4, sk=4, n_head=2, n_head_kv=1,
                         head_dim=300)
    assert ca.lib.ca_attention_dev(ctypes.byref(a), None) == ca.CA_ERR_UNSUPPORTED
    a = ca.make_dev_args(fake, fake, fake, fake, batch=1, sq=4, sk=4, n_head=3, n_head_kv=2,
                         head_dim=128)
    assert ca.lib.ca_attention_dev(ctypes.byref(a), None) == ca.CA_ERR_INVALID
    a = ca.make_dev_args(fake + 2, fake, fake, fake, batch=1, sq=4, sk=4, n_head=2,
                         n_head_kv=1, head_dim=128)
    assert ca.lib.ca_attention_dev(ctypes.byref(a), None) == ca.CA_ERR_INVALID
    # Empty batches are a no-op success.
    a = ca.make_dev_args(fake, fake, fake, fake, batch=0, sq=4, sk=4, n_head=2, n_head_kv=1,
                         head_dim=128)
    assert ca.lib.ca_attention_dev(ctypes.byref(a), None) == ca.CA_OK


def test_block_entry_rejects_bad_arguments():
    a = ca.make_block_args(None, None, None, batch=1, n_active=1, active_pos=None, rope=None,
                           rope_len=1, rope_dim=2, cache_k=None, cache_v=None, n_total=1,
                           q_work=None, out=None, n_head=1, n_head_kv=1, head_dim=8)
    assert ca.lib.ca_attention_block_dev(ctypes.byref(a), None) == ca.CA_ERR_INVALID


def test_host_entry_validates_shape():
    s = ca.AttnShape(nq=2, nk=2, n_head=3, n_head_kv=2, head_dim=8)
    out = np.zeros(2 * 3 * 8, np.float32)
    q = np.zeros(2 * 3 * 8, np.float32)
    k = np.zeros(2 * 2 * 8, np.float32)
    cs = s.to_c()
    cq, _k1 = ca.Rows([0, 1]).to_c()
    ck, _k2 = ca.Rows([0, 1]).to_c()
    rc = ca.lib.ca_attention_host_f32(out.ctypes.data, q.ctypes.data, k.ctypes.data,
                                      k.ctypes.data, ctypes.byref(cs), ctypes.byref(cq),
                                      ctypes.byref(ck))
    assert rc == ca.CA_ERR_INVALID


def test_selftest_rejects_bad_limits_without_launching():
    assert ca.lib.ca_selftest_wait_timeout(0, None) == ca.CA_ERR_INVALID
    assert ca.lib.ca_selftest_wait_timeout(-5, None) == ca.CA_ERR_INVALID
    assert ca.lib.ca_selftest_wait_timeout(2_000_000_000, None) == ca.CA_ERR_INVALID


def test_host_bf16_rounding_is_round_to_nearest_even():
    """ca_round_bf16_host (the rounding the host-buffer entry point applies
    before its copies) against torch's round-to-nearest-even on the CPU:
    ties, values just below and above ties, subnormals, the overflow edge,
    infinities; every NaN becomes 0x7FFF (what cvt.rn.bf16.f32 gives)."""
    import numpy as np
    import torch
    rng = np.random.default_rng(3)
    bits = rng.integers(0, 2**32, size=1_000_003, dtype=np.uint64).astype(np.uint32)
    edge = np.array([0x3f808000, 0x3f818000, 0x3f807fff, 0x3f808001, 0x00000001, 0x00008000,
                     0x00018000, 0x7f7fffff, 0x7f7f8000, 0x7f7f7fff, 0xff7fffff, 0x7f800000,
                     0xff800000, 0x00000000, 0x80000000, 0x7fc00000, 0xffc00001, 0x7f800001],
                    dtype=np.uint32)
    bits = np.concatenate([edge, bits])
    x = bits.view(np.float32)
    got = ca.round_bf16_host(x)
    want = torch.from_numpy(x.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], want[~nan])
    assert np.all(got[nan] == 0x7FFF)
    # Small calls (one task on the calling thread) round the same way.
    assert np.array_equal(ca.round_bf16_host(x[:1000]), got[:1000])
