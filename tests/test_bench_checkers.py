"""The float64 checkers bench.py uses on the device (its parity figures for
the prefill, long-context, backward and gated workloads) against the oracle,
on the CPU at small sizes: the bench's max_rel_err values are only as good as
these restatements."""
import numpy as np
import torch

from oracle import retention_ref as R

HD = 256


def _weights(rng, d, n):
    return [0.05 * rng.standard_normal((d, d)) for _ in range(n)]


def test_rows_reference_matches_oracle_forward():
    """bench.msr_rows_reference (row blocks, state formed in one product)
    equals the oracle's parallel-form MultiScaleRetention forward
    (aceflow/nn/retention.py:44-66), whole rows and a column range."""
    from bench import msr_rows_reference

    rng = np.random.default_rng(3)
    T, H = 200, 2
    d = H * HD
    x = rng.standard_normal((1, T, d))
    wq, wk, wv, wo = _weights(rng, d, 4)
    rw = 1 + 0.1 * rng.standard_normal(d)
    ref = R.msr_forward64(x, wq, wk, wv, wo, H, rw, 1e-6)[0]
    rows = [(0, 64), (100, 164), (136, 200)]
    t = torch.from_numpy
    got = msr_rows_reference(t(x[0]), t(np.concatenate([wq, wk, wv])), t(wo), t(rw), H, 1e-6, rows)
    for (r0, r1), g in zip(rows, got):
        np.testing.assert_allclose(g.numpy(), ref[r0:r1], rtol=1e-9, atol=1e-9)
    part = msr_rows_reference(t(x[0]), t(np.concatenate([wq, wk, wv])), t(wo), t(rw), H, 1e-6, rows[1:2],
                              col_range=(128, 384))
    np.testing.assert_allclose(part[0].numpy(), ref[100:164, 128:384], rtol=1e-9, atol=1e-9)


def test_rows_reference_gated_matches_oracle():
    """The gated form of the checker (swish gate, per-head GroupNorm) equals
    the oracle's msr_gated_forward64."""
    from bench import msr_rows_reference

    rng = np.random.default_rng(4)
    T, H = 150, 2
    d = H * HD
    x = rng.standard_normal((1, T, d))
    wq, wk, wv, wg, wo = _weights(rng, d, 5)
    ref, _ = R.msr_gated_forward64(x, wq, wk, wv, wg, wo, H, None, None, 1e-6)
    rows = [(0, 50), (100, 150)]
    t = torch.from_numpy
    got = msr_rows_reference(t(x[0]), t(np.concatenate([wq, wk, wv])), t(wo), t(np.ones(d)), H, 1e-6, rows,
                             w_g=t(wg))
    for (r0, r1), g in zip(rows, got):
        np.testing.assert_allclose(g.numpy(), ref[0, r0:r1], rtol=1e-9, atol=1e-9)


def test_backward_blocks_reference_matches_oracle():
    """bench.backward_blocks_reference's dQ (first rows) and dK, dV (last
    rows) equal the oracle's closed-form gradients of the whole stream."""
    from bench import backward_blocks_reference

    rng = np.random.default_rng(5)
    T, H, n = 300, 2, 64
    d = H * HD
    qkv = rng.standard_normal((T, 3 * d))
    dout = rng.standard_normal((T, d))
    sh = lambda a: a.reshape(1, T, H, HD).transpose(0, 2, 1, 3)  # noqa: E731
    q, k, v = (sh(qkv[:, i * d:(i + 1) * d]) for i in range(3))
    dq, dk, dv, _ = R.retention_backward64(q, k, v, R.gammas(H), sh(dout))
    blocks = backward_blocks_reference(torch.from_numpy(qkv), torch.from_numpy(dout), d, (0, 1), T, n)
    for h in range(H):
        np.testing.assert_allclose(blocks[(h, "dq")].numpy(), dq[0, h, :n], rtol=1e-9, atol=1e-9)
        np.testing.assert_allclose(blocks[(h, "dk")].numpy(), dk[0, h, T - n:], rtol=1e-9, atol=1e-9)
        np.testing.assert_allclose(blocks[(h, "dv")].numpy(), dv[0, h, T - n:], rtol=1e-9, atol=1e-9)
