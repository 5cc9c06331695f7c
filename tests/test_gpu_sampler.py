"""GPU parity of the denoising step's per-candidate statistics
(ca_candidate_stats: collect_candidates with the greedy pick,
src/model/sampler.rs:720-764, after suppress_mask_token / suppress_tokens
:90-113) against the oracle's sequential restatement, and one whole
process_logits step of the host mirror against the same step built on the
oracle's statistics.

Bar: token and margin exact (margin is one subtraction of two exact
maxima); entropy within 1e-4 absolute + 1e-4 relative. prob = exp(top1 -
log_sum_exp) inherits the relative error of the row's sum of exponentials,
which the reference folds sequentially in f32: over 10^5 terms that sum
itself is off by up to ~5e-4 relative. So prob must lie within 1e-5 + 2e-3
relative of the oracle AND be at least as close to the float64 value as the
oracle is (to 1e-6)."""
import numpy as np
import pytest
import torch

from canvas_attn import denoise as dn
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _logits(g, rows, vocab, scale=3.0):
    return (torch.randn(rows, vocab, generator=g) * scale).numpy().astype(np.float32)


def _gpu_stats(lg, rows, *, mask_id=-1, suppress=(), row_stride=0, want_prob=True):
    n_rows, vocab = lg.shape
    if row_stride:
        buf = np.full((n_rows, row_stride), 7.0, np.float32)  # padding must not be read
        buf[:, :vocab] = lg
        d = torch.from_numpy(buf).cuda()
    else:
        d = torch.from_numpy(lg.copy()).cuda()
    r = torch.tensor(rows, dtype=torch.int32, device="cuda")
    n = len(rows)
    tok = torch.empty(n, dtype=torch.int32, device="cuda")
    ent, mar, prob = (torch.full((n,), float("nan"), device="cuda") for _ in range(3))
    sup = torch.tensor(list(suppress), dtype=torch.int32, device="cuda") if suppress else None
    dn.candidate_stats(d, r, tok, ent, mar, prob, n_vocab=vocab, row_stride=row_stride,
                       mask_id=mask_id, suppress=sup, want_entropy=True, want_prob=want_prob)
    torch.cuda.synchronize()
    return (tok.cpu().numpy(), ent.cpu().numpy(), mar.cpu().numpy(), prob.cpu().numpy(),
            d.cpu().numpy()[:, :vocab])


def _prob64(lg, rows, mask_id=-1, suppress=()):
    """exp(top1 - log_sum_exp) of each row in float64, after suppression."""
    x = np.array(lg, dtype=np.float64)
    for i in [mask_id, *suppress]:
        if 0 <= i < x.shape[1]:
            x[:, i] = -np.inf
    out = []
    for r in rows:
        m = x[r].max()
        out.append(np.exp(m - (m + np.log(np.exp(x[r] - m).sum()))))
    return np.array(out)


def _check(got, ref, what, p64=None):
    tok, ent, mar, prob = got[:4]
    rt, re_, rm, rp = ref
    np.testing.assert_array_equal(tok, rt, err_msg=f"{what}: token")
    np.testing.assert_array_equal(mar, rm, err_msg=f"{what}: margin")
    np.testing.assert_allclose(ent, re_, atol=1e-4, rtol=1e-4, err_msg=f"{what}: entropy")
    np.testing.assert_allclose(prob, rp, atol=1e-5, rtol=2e-3, err_msg=f"{what}: prob")
    if p64 is not None:
        assert (np.abs(prob - p64) <= np.abs(rp - p64) + 1e-6).all(), f"{what}: prob vs f64"


@pytest.mark.parametrize("vocab,row_stride", [(16, 0), (1001, 0), (126464, 0),
                                              (151936, 152064), (262144, 0)])
def test_candidate_stats_match_oracle(vocab, row_stride):
    g = torch.Generator().manual_seed(vocab)
    n_rows = 24
    lg = _logits(g, n_rows, vocab)
    rows = [0, 3, 5, 6, 11, 12, 20, 23]
    mask_id, suppress = vocab - 1, (1, 2, vocab // 2)
    got = _gpu_stats(lg, rows, mask_id=mask_id, suppress=suppress, row_stride=row_stride)
    ref = orc.candidate_stats(lg, rows, mask_id=mask_id, suppress=suppress)
    _check(got, ref, f"vocab {vocab}", _prob64(lg, rows, mask_id, suppress))
    # Suppressed entries of the candidate rows are -inf in the buffer afterwards.
    after = got[4]
    assert np.isneginf(after[rows][:, [1, 2, vocab // 2, vocab - 1]]).all()


def test_candidate_stats_edge_rows():
    vocab = 4099
    lg = np.zeros((5, vocab), np.float32)
    lg[0, [7, 900, 4000]] = 5.0           # tied maxima: first index, margin 0
    lg[1, :] = -np.inf
    lg[1, 4098] = 1.0                     # one finite entry: margin +inf, entropy 0
    lg[2, :] = -np.inf                    # nothing finite: token 0
    lg[3, 10] = 100.0                     # peaked
    lg[4, :] = np.linspace(-30, 30, vocab, dtype=np.float32)
    rows = [0, 1, 3, 4]
    got = _gpu_stats(lg, rows)
    ref = orc.candidate_stats(lg, rows)
    _check(got, ref, "edge rows")
    assert got[0][0] == 7 and got[2][0] == 0.0 and np.isposinf(got[2][1])
    tok = _gpu_stats(lg, [2])[0]
    assert tok[0] == 0


@pytest.mark.parametrize("remasking", [dn.LOW_CONFIDENCE, dn.MARGIN, dn.CONFIDENCE,
                                       dn.ENTROPY_EXIT, dn.ENTROPY_BOUND])
def test_process_logits_step_matches_oracle_step(remasking):
    # A 64-position canvas (16 prompt tokens, 48 masked), vocab 32000, logit
    # shift 1 (Dream-style), one suppressed id; the GPU step must commit the
    # same positions and tokens as the same step on the oracle's statistics.
    g = torch.Generator().manual_seed(100 + remasking)
    L, P, vocab, mask_id, shift = 64, 16, 32000, 31999, 1
    lg = _logits(g, L, vocab, scale=4.0)
    seq = [int(x) for x in torch.randint(0, 1000, (P,), generator=g)] + [mask_id] * (L - P)
    masked = [False] * P + [True] * (L - P)
    params = dn.StepParams(remasking=remasking, confidence_threshold=0.3,
                           entropy_threshold=2.0, eb_entropy_bound=2.5, suppress_ids=[5])
    st = dn.DenoiseState(seq, masked, mask_id)
    n = dn.process_logits(st, torch.from_numpy(lg.copy()).cuda(), vocab, range(P, L), shift,
                          2, 8, params)
    # The same step on the oracle's statistics.
    pos = list(range(P, L))
    tok, ent, mar, prob = orc.candidate_stats(lg, [p - shift for p in pos], mask_id=mask_id,
                                              suppress=[5])
    cands = [dn.Candidate(p, int(tok[i]), float(ent[i]), float(mar[i]), float(prob[i]))
             for i, p in enumerate(pos)]
    ref = dn.DenoiseState(seq, masked, mask_id)
    k = dn.rank_candidates(cands, params, 2, 8)
    m = dn.commit(ref, cands, k, params)
    assert n == m and n > 0
    np.testing.assert_array_equal(st.seq, ref.seq)
    np.testing.assert_array_equal(st.is_masked, ref.is_masked)
