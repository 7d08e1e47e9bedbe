"""Sampling kernel (af_sample_rows) against the oracle's restatement of the
reference's sample_token_from_logits (aceflow-core/src/cpu/sampler.rs:83-180).

The kernel's sums are fp32 block reductions, the reference's sequential: a
draw (or top_p) within 1e-4 of a running-sum boundary may land on the
neighbouring token, so such rows are not compared (the oracle reports the
margin); all other rows must give the same token.
"""
import numpy as np
import pytest
import torch

from oracle import retention_ref as R

pytestmark = pytest.mark.gpu

MARGIN = 1e-4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _sample(dev, logits, u, ctx, t, k, p, rp):
    from aceflow_b200 import cuda_ops

    lt = torch.as_tensor(np.asarray(logits, np.float32)).to(dev)
    ut = None if u is None else torch.as_tensor(np.asarray(u, np.float32)).to(dev)
    ct = None if ctx is None else torch.as_tensor(np.asarray(ctx, np.int32)).to(dev)
    out = cuda_ops.sample_rows(lt, ut, ct, temperature=t, top_k=k, top_p=p, repetition_penalty=rp)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_kat_reference_sampler_tests(dev):
    """sampler.rs:187-197 through the GPU (greedy, penalty)."""
    assert _sample(dev, [[1.0, 3.0, 2.0]], None, None, 0.0, 0, 1.0, 1.0)[0] == 1
    assert _sample(dev, [[1.0, 3.0, 2.0]], None, [[1]], 0.0, 0, 1.0, 10.0)[0] == 2
    assert _sample(dev, [[5.0, 5.0, 1.0]], None, None, 0.0, 0, 1.0, 1.0)[0] == 0


def test_hand_worked_draws(dev):
    """Probabilities .1 .2 .3 .4: draws map to tokens 3, 2, 1, 0 by running
    sums .4 .7 .9 1; top-k, top-p and a penalised tie in index order."""
    lg = np.log(np.array([1.0, 2.0, 3.0, 4.0], np.float32))
    us = [0.0, 0.39, 0.41, 0.69, 0.71, 0.89, 0.91]
    got = _sample(dev, np.tile(lg, (len(us), 1)), us, None, 1.0, 0, 1.0, 1.0)
    assert got.tolist() == [3, 3, 2, 2, 1, 1, 0]
    assert _sample(dev, [lg, lg], [0.56, 0.58], None, 1.0, 2, 1.0, 1.0).tolist() == [3, 2]
    assert _sample(dev, [lg, lg], [0.99, 0.99], None, 1.0, 0, 1.0, 1.0).tolist() == [0, 0]
    assert _sample(dev, [lg], [0.99], None, 1.0, 0, 0.5, 1.0).tolist() == [2]
    assert _sample(dev, [lg], [0.99], None, 1.0, 0, 0.3, 1.0).tolist() == [3]
    assert _sample(dev, [lg, lg], [0.5, 0.7], [[3, 3], [3, 3]], 1.0, 0, 1.0, 2.0).tolist() == [1, 3]


def test_equal_logits_lowest_index_first(dev):
    """All logits equal, top_k 5: tokens 0..4, each with probability 0.2."""
    z = np.zeros((5, 1000), np.float32)
    us = [0.05, 0.25, 0.45, 0.65, 0.85]
    assert _sample(dev, z, us, None, 1.0, 5, 1.0, 1.0).tolist() == [0, 1, 2, 3, 4]
    assert [R.sample_token(z[0], (), 1.0, 5, 1.0, 1.0, u) for u in us] == [0, 1, 2, 3, 4]


@pytest.mark.parametrize("t,k,p,rp", [(0.7, 40, 0.9, 1.2), (1.0, 0, 1.0, 1.0), (1.3, 0, 0.95, 1.0),
                                      (0.5, 1000, 0.5, 1.5), (1.0, 1, 1.0, 1.0), (2.0, 50, 1.0, 1.1),
                                      (1.0, 0, 0.0, 1.0), (0.8, 32000, 0.99, 1.0), (0.0, 40, 0.9, 1.2)])
def test_matches_oracle_vocab_32000(dev, t, k, p, rp):
    """32 rows of a 32000-token vocabulary (the configured model's), random
    logits and contexts (repeats, -1 padding, out-of-range ids), draws in
    [0, 1) including 0: the same token as the oracle wherever the result does
    not hinge on rounding."""
    rng = np.random.default_rng(int(t * 100) + k + int(p * 10) + int(rp * 10))
    rows, V = 32, 32000
    logits = (3.0 * rng.standard_normal((rows, V))).astype(np.float32)
    ctx = rng.integers(0, V, (rows, 60)).astype(np.int32)
    ctx[:, :10] = ctx[:, 10:20]  # repeated ids are penalised once
    ctx[:, -5:] = -1              # padding
    ctx[0, 0] = 40000             # out of range: ignored
    logits[:, ctx[1, 20]] = 25.0  # a penalised id that would otherwise dominate row 1
    u = rng.random(rows).astype(np.float32)
    u[0] = 0.0
    got = _sample(dev, logits, u, ctx, t, k, p, rp)
    compared = 0
    for r in range(rows):
        want, margin = R.sample_token(logits[r], ctx[r], t, k, p, rp, float(u[r]), detail=True)
        if margin < MARGIN:
            continue
        compared += 1
        assert got[r] == want, (r, got[r], want, margin)
    assert compared >= rows * 3 // 4
