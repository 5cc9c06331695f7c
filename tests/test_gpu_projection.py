"""GPU parity of the projections around attention (src/model/forward.rs:
275-294, :345-350): the dequantisers against the oracle's restatement of
src/kernels.rs (fp32 output bit-identical, bf16 output = the oracle's value
rounded once), the embedding gather, and the linear layer (bf16 operands,
fp32 accumulation) against a float64 product of the same bf16 operands and
against the reference's own Q8_K-activation product."""
import numpy as np
import pytest
import torch

from canvas_attn import projection as pj
from oracle import oracle as orc
from quant_helpers import random_rows

pytestmark = pytest.mark.gpu

QTYPES = [orc.QTYPE_Q4_K, orc.QTYPE_Q6_K, orc.QTYPE_Q4_0, orc.QTYPE_Q8_0, orc.QTYPE_F16]


@pytest.mark.parametrize("qtype", QTYPES)
def test_dequantize_bit_exact(qtype):
    rows, cols = 48, 1024
    w = random_rows(qtype, rows, cols, seed=qtype)
    ref = orc.dequantize(qtype, w, rows, cols)
    src = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    out32 = torch.empty(rows, cols, device="cuda")
    out16 = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
    pj.dequantize(qtype, src, rows, cols, out32, dst_f32=True)
    pj.dequantize(qtype, src, rows, cols, out16)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out32.cpu().numpy(), ref)
    want16 = torch.from_numpy(ref).to(torch.bfloat16)
    assert torch.equal(out16.cpu(), want16)


@pytest.mark.parametrize("qtype", [orc.QTYPE_Q4_K, orc.QTYPE_Q6_K, orc.QTYPE_Q8_0])
def test_embedding_gather(qtype):
    # embed_tokens (forward.rs:175-246) with Gemma's embed scale applied after.
    n_vocab, cols = 300, 512
    table = random_rows(qtype, n_vocab, cols, seed=7 + qtype)
    ref_all = orc.dequantize(qtype, table, n_vocab, cols)
    tokens = np.array([5, 299, 0, 5, 123, 42], np.int32)
    scale = np.float32(np.sqrt(np.float32(cols)))
    out = torch.full((len(tokens), cols), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    pj.embed(qtype, torch.from_numpy(np.ascontiguousarray(table)).cuda(), n_vocab, cols,
             torch.from_numpy(tokens).cuda(), out, scale=float(scale), status=status)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref_all[tokens] * scale)
    assert int(status.item()) == 0
    # An out-of-range id skips its row and reports through the status word.
    bad = torch.tensor([1, 300], dtype=torch.int32, device="cuda")
    out2 = torch.zeros(2, cols, device="cuda")
    pj.embed(qtype, torch.from_numpy(np.ascontiguousarray(table)).cuda(), n_vocab, cols, bad,
             out2, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1 and (out2[1] == 0).all()


@pytest.mark.parametrize("qtype,out_f32", [(orc.QTYPE_Q4_K, True), (orc.QTYPE_Q6_K, True),
                                           (orc.QTYPE_Q4_K, False)])
def test_linear_with_bias_and_residual(qtype, out_f32):
    n, rows, cols = 100, 384, 1024
    g = torch.Generator().manual_seed(qtype + int(out_f32))
    w = random_rows(qtype, rows, cols, seed=100 + qtype)
    wd = torch.empty(rows, cols, dtype=torch.bfloat16, device="cuda")
    pj.dequantize(qtype, torch.from_numpy(np.ascontiguousarray(w)).cuda(), rows, cols, wd)
    act = torch.randn(n, cols, generator=g)
    bias = torch.randn(rows, generator=g)
    odt = torch.float32 if out_f32 else torch.bfloat16
    res = torch.randn(n, rows, generator=g).to(odt)
    out = torch.empty(n, rows, device="cuda", dtype=odt)
    act_b = act.to(torch.bfloat16)
    pj.linear(act_b.cuda(), wd, out, n=n, rows=rows, cols=cols, bias=bias.cuda(),
              residual=res.cuda())
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().astype(np.float64)
    # float64 product of the same bf16 operands
    exact = (act_b.double().numpy() @ wd.double().cpu().numpy().T + bias.double().numpy()
             + res.double().numpy())
    tol = 1e-5 if out_f32 else 4e-3
    scale = np.abs(exact).max()
    assert np.abs(got - exact).max() <= tol * scale, np.abs(got - exact).max() / scale
    # Against the reference's own arithmetic (activations quantised to Q8_K,
    # src/model/matmul.rs:90-110): within that quantisation's error.
    ref = orc.linear_q8k(qtype, w, rows, cols, act.numpy()) + bias.numpy() + res.float().numpy()
    num = np.sqrt(((got - ref) ** 2).sum(axis=1))
    den = np.sqrt(((ref - res.float().numpy() - bias.numpy()) ** 2).sum(axis=1))
    assert (num / den).max() < 2e-2, (num / den).max()
