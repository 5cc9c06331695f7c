"""Failure detection on the GPU without a GPU fault.

Every pipeline wait of the attention kernel is bounded: when it expires the
kernel stores CA_ERR_TIMEOUT in a device error word and returns instead of
hanging. ca_selftest_wait_timeout runs that same bounded wait on an mbarrier
nothing arrives on (a flag that nobody sets), with a short limit. The test
checks that the expiry is reported once, that the status word is cleared by
the read, and that the context still runs attention correctly afterwards."""
import time

import pytest
import torch

import canvas_attn as ca
from helpers import bf16_round, check_close, oracle_attention, randn

pytestmark = pytest.mark.gpu


def _small_attention():
    g = torch.Generator().manual_seed(11)
    q = bf16_round(randn(g, 1, 40, 2, 64))
    k = bf16_round(randn(g, 1, 40, 1, 64))
    v = bf16_round(randn(g, 1, 40, 1, 64))
    out = torch.empty((1, 40, 2, 64), dtype=torch.float32, device="cuda")
    ca.attention_dev(q.to(torch.bfloat16).cuda(), k.to(torch.bfloat16).cuda(),
                     v.to(torch.bfloat16).cuda(), out, batch=1, sq=40, sk=40, n_head=2,
                     n_head_kv=1, head_dim=64, out_f32=True, scale=0.125)
    return q, k, v, out


def test_expired_wait_is_reported_and_context_survives():
    torch.cuda.init()
    assert ca.device_status() == ca.CA_OK
    t0 = time.perf_counter()
    ca.selftest_wait_timeout(20_000_000)  # 20 ms
    assert ca.device_status() == ca.CA_ERR_TIMEOUT
    waited = time.perf_counter() - t0
    assert 0.015 < waited < 5.0
    assert ca.device_status() == ca.CA_OK  # read-and-clear
    # The context is intact: a normal call right after gives correct results.
    q, k, v, out = _small_attention()
    assert ca.device_status() == ca.CA_OK
    ref = oracle_attention(q[0].numpy(), k[0].numpy(), v[0].numpy(), nq=40, nk=40, h=2, hkv=1,
                           hd=64, scale=0.125)
    check_close(out[0].cpu().numpy(), ref, 2, 64, what="after expiry")


def test_expiry_on_a_side_stream():
    s = torch.cuda.Stream()
    ca.selftest_wait_timeout(5_000_000, stream=s)
    assert ca.device_status(stream=s) == ca.CA_ERR_TIMEOUT
    assert ca.device_status(stream=s) == ca.CA_OK


def test_expiry_reported_to_a_per_call_status_word():
    # A launch given its own status word reports there, not in the device-wide
    # word: another stream polling ca_device_status neither sees nor clears it.
    assert ca.device_status() == ca.CA_OK
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    ca.selftest_wait_timeout_status(5_000_000, word, stream=s)
    s.synchronize()
    assert ca.device_status() == ca.CA_OK
    assert int(word.item()) == ca.CA_ERR_TIMEOUT
    # An attention call with a status word leaves it at 0 when nothing expires.
    word.zero_()
    g = torch.Generator().manual_seed(12)
    q = bf16_round(randn(g, 1, 40, 2, 64)).to(torch.bfloat16).cuda()
    k = bf16_round(randn(g, 1, 40, 1, 64)).to(torch.bfloat16).cuda()
    out = torch.empty((1, 40, 2, 64), dtype=torch.float32, device="cuda")
    ca.attention_dev(q, k, k, out, batch=1, sq=40, sk=40, n_head=2, n_head_kv=1, head_dim=64,
                     out_f32=True, scale=0.125, status=word)
    torch.cuda.synchronize()
    assert int(word.item()) == ca.CA_OK
    assert ca.device_status() == ca.CA_OK
