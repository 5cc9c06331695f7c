"""The denoising step's CPU side: the oracle's restatement of the sampler's
statistics pinned to the reference's own tests (src/model/tests.rs), the
C-ABI tokens_to_unmask against that restatement, and the host mirror's
ranking / commit logic (src/model/sampler.rs:597-671) on hand-built
candidates. No GPU needed."""
import numpy as np

from canvas_attn import denoise as dn
from oracle import oracle as orc


def test_oracle_entropy_and_top2_known_answers():
    # tests.rs:27-37: uniform 16 -> ln 16; one logit at 100 -> ~0.
    assert abs(orc.compute_entropy(np.zeros(16)) - np.log(16)) < 1e-5
    row = np.zeros(16, np.float32)
    row[3] = 100.0
    assert orc.compute_entropy(row) < 1e-3
    # tests.rs:281-284
    assert orc.top2_logits([1.0, 5.0, 3.0, 5.0]) == (5.0, 5.0)
    assert orc.top2_logits([2.0, -1.0]) == (2.0, -1.0)
    # tests.rs:287-293: lse([0, 0]) = ln 2, p(top1) = 0.5
    lse = orc.log_sum_exp([0.0, 0.0])
    assert abs(lse - np.log(2)) < 1e-6
    assert abs(np.exp(0.0 - lse) - 0.5) < 1e-6


def test_schedule_unmasks_everything():
    # tests.rs:13-24, through the C ABI.
    for schedule in (dn.COSINE, dn.LINEAR):
        for total in (1, 4, 16):
            masked = 128
            for step in range(total):
                masked -= dn.tokens_to_unmask(step, total, masked, schedule)
            assert masked == 0


def test_tokens_to_unmask_matches_oracle():
    for schedule in (dn.COSINE, dn.LINEAR):
        for total in (1, 2, 3, 7, 16, 64):
            for masked in (0, 1, 5, 31, 128, 1000):
                for step in range(total + 1):
                    assert dn.tokens_to_unmask(step, total, masked, schedule) == \
                        orc.tokens_to_unmask(step, total, masked, schedule)


def _cands(vals):
    return [dn.Candidate(pos=i, token=100 + i, entropy=e, margin=m, prob=p)
            for i, (e, m, p) in enumerate(vals)]


def test_rank_candidates_orders_and_counts():
    vals = [(0.5, 1.0, 0.95), (0.1, 3.0, 0.5), (0.5, 2.0, 0.99), (2.0, 0.0, 0.2)]
    # LowConfidence: ascending entropy, stable for ties; cosine schedule count.
    c = _cands(vals)
    n = dn.rank_candidates(c, dn.StepParams(remasking=dn.LOW_CONFIDENCE), 0, 4)
    assert [x.pos for x in c] == [1, 0, 2, 3]
    assert n == dn.tokens_to_unmask(0, 4, 4, dn.COSINE)
    # Margin: descending margin.
    c = _cands(vals)
    dn.rank_candidates(c, dn.StepParams(remasking=dn.MARGIN), 0, 4)
    assert [x.pos for x in c] == [1, 2, 0, 3]
    # Confidence: descending prob; all with prob >= threshold are committed.
    c = _cands(vals)
    n = dn.rank_candidates(c, dn.StepParams(remasking=dn.CONFIDENCE,
                                            confidence_threshold=0.9), 3, 4)
    assert [x.pos for x in c] == [2, 0, 1, 3] and n == 4  # last step: schedule takes all
    c = _cands(vals)
    n = dn.rank_candidates(c, dn.StepParams(remasking=dn.CONFIDENCE,
                                            confidence_threshold=0.9), 0, 16)
    assert n == 2
    # EntropyExit: schedule minimum raised to the easy count.
    c = _cands(vals)
    n = dn.rank_candidates(c, dn.StepParams(remasking=dn.ENTROPY_EXIT,
                                            entropy_threshold=0.6), 0, 64)
    assert n == 3
    # EntropyBound: at least one, else those below the bound.
    c = _cands(vals)
    assert dn.rank_candidates(c, dn.StepParams(remasking=dn.ENTROPY_BOUND,
                                               eb_entropy_bound=0.05), 0, 4) == 1
    # total_cmp order: -0.0 before +0.0.
    c = _cands([(0.0, 0, 0), (-0.0, 0, 0)])
    dn.rank_candidates(c, dn.StepParams(remasking=dn.LOW_CONFIDENCE), 0, 4)
    assert [x.pos for x in c] == [1, 0]


def test_commit_and_credit():
    st = dn.DenoiseState([7, 9, 9, 9, 9], [False, True, True, True, True], mask_id=9)
    params = dn.StepParams(credit_steps=2)
    for step in range(3):
        cands = [dn.Candidate(p, 40 + p, 1.0, 0.0, 0.0) for p in (1, 2, 3, 4) if st.is_masked[p]]
        dn.update_credit(st, cands, params)
        n = dn.commit(st, cands, 1 if step == 0 else 0, params)
        if step == 0:
            assert n == 1 and not st.is_masked[1] and st.seq[1] == 41
        elif step == 1:
            assert n == 0  # credit 1 < 2
        else:
            assert n == 3  # credit reached 2 for the stable picks
    assert st.n_masked == 0 and list(st.seq) == [7, 41, 42, 43, 44]
