"""Decoder stack (AceEngine twin) parity against the C restatement of
AceEngine (oracle/cpu_ref.c: forward_layer_internal + greedy generation).

fp32 weights: logits within 1e-4 relative and identical greedy tokens.
bf16 weights: the oracle runs on the same bf16-rounded weights in fp32;
logits within 2e-2 under teacher forcing (oracle tokens fed back), so one
near-tie cannot cascade.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import cpu_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _model(L, d, f, V, seed, bf16):
    rng = np.random.default_rng(seed)
    r = (lambda a: torch.from_numpy(a).bfloat16().float().numpy()) if bf16 else (lambda a: a)
    layers = []
    for _ in range(L):
        layers.append(dict(
            w_qkv=r((0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)),
            w_o=r((0.02 * rng.standard_normal((d, d))).astype(np.float32)),
            w_gate_up=r((0.02 * rng.standard_normal((2 * f, d))).astype(np.float32)),
            w_down=r((0.02 * rng.standard_normal((d, f))).astype(np.float32)),
            norm1=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
            norm2=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
            ret_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32)))
    emb = r(rng.standard_normal((V, d)).astype(np.float32))
    return layers, emb


def _engine(layers, emb, H, B, dtype, eps):
    from aceflow_b200.engine import AceEngine

    L = len(layers)
    d = emb.shape[1]
    eng = AceEngine(L, d, H, emb, batch=B, weight_dtype=dtype, eps=eps)
    for i, w in enumerate(layers):
        eng.load_layer_weights(i, w["w_qkv"], w["w_o"], w["w_gate_up"], w["w_down"], w["norm1"], w["norm2"],
                               w["ret_norm"])
    return eng


def test_forward_layer_fp32_matches_oracle(dev):
    L, d, H, f, V, B = 1, 256, 2, 96, 50, 3
    layers, emb = _model(L, d, f, V, 1, False)
    eng = _engine(layers, emb, H, B, "float32", 1e-5)
    rng = np.random.default_rng(5)
    states = np.zeros((B, L, H, d // H, d // H), np.float32)
    for _ in range(4):
        x = rng.standard_normal((B, d)).astype(np.float32)
        ref = cpu_ref.forward_layer(x.copy(), layers, 0, states, np.array(
            [1 - 2.0 ** (-5 - h) for h in range(H)], np.float32), 1e-5)
        got = eng.forward_layer(0, x.copy())
        assert rel_err(got, ref) < 1e-4


@pytest.mark.parametrize("dtype,shape", [("float32", (2, 512, 2, 256, 300, 3, 20, 6)),
                                         ("bfloat16", (2, 512, 2, 256, 300, 3, 20, 6)),
                                         ("bfloat16", (1, 1024, 4, 512, 500, 64, 6, 3)),
                                         ("bfloat16", (1, 1024, 4, 512, 500, 100, 4, 2))])
def test_generate_matches_oracle(dev, dtype, shape):
    """Prefill + greedy decode; bf16 weights with up to 256 streams take the
    transposed decode projections (batch 3, 64, 100 -> tiles 16, 64, 128)."""
    bf16 = dtype == "bfloat16"
    L, d, H, f, V, B, P, n = shape
    layers, emb = _model(L, d, f, V, 2, bf16)
    rng = np.random.default_rng(9)
    prompts = rng.integers(0, V, (B, P)).astype(np.int32)
    toks_ref, logits_ref, _, _ = cpu_ref.generate_greedy(layers, emb, prompts, n, H, 1e-6, want_logits=True)
    eng = _engine(layers, emb, H, B, dtype, 1e-6)
    toks, logits = eng.generate_batch(prompts, n, teacher=toks_ref, return_logits=True)
    tol = 2e-2 if bf16 else 1e-4
    assert rel_err(logits, logits_ref) < tol
    if not bf16:
        assert np.array_equal(toks, toks_ref)
    else:
        top2 = np.sort(logits_ref, -1)[..., -2:]
        clear = (top2[..., 1] - top2[..., 0]) > 0.05 * np.abs(logits_ref).max()
        assert np.array_equal(toks[clear], toks_ref[clear])


def test_generate_stream_api(dev):
    L, d, H, f, V = 1, 256, 1, 64, 40
    layers, emb = _model(L, d, f, V, 4, False)
    eng = _engine(layers, emb, H, 1, "float32", 1e-5)
    out = eng.generate_stream([3, 7, 1], 5, temperature=0.0, repetition_penalty=1.0)
    ref, _, _, _ = cpu_ref.generate_greedy(layers, emb, np.array([[3, 7, 1]], np.int32), 5, H, 1e-5,
                                           stop_at_eos=True)
    exp = []
    for t in ref[0]:
        if t < 0:
            break
        exp.append(int(t))
        if t == 2:
            break
    assert out == exp
    # the reference's defaults (temperature 0.7, top_k 40, top_p 0.9, penalty 1.2) sample on the
    # GPU; a seed makes the draws repeatable
    eng.reset_memory()
    a1 = eng.generate_stream([1, 5], 4, seed=11)
    eng.reset_memory()
    a2 = eng.generate_stream([1, 5], 4, seed=11)
    assert a1 == a2 and 1 <= len(a1) <= 4 and all(0 <= t < V for t in a1)


def test_generate_sampling_matches_oracle(dev):
    """Sampled generation (temperature, top-k, top-p, repetition penalty over
    the last 60 ids of prompt + output): each step's token is the oracle's
    sample_token on that step's logits, context window and draw (rows whose
    draw lies within rounding of a boundary are not compared)."""
    from oracle import retention_ref as R

    L, d, H, f, V, B, P, n = 1, 256, 2, 96, 300, 3, 58, 6
    layers, emb = _model(L, d, f, V, 9, False)
    eng = _engine(layers, emb, H, B, "float32", 1e-5)
    rng = np.random.default_rng(2)
    prompts = rng.integers(3, V, (B, P)).astype(np.int32)
    uni = rng.random((B, n)).astype(np.float32)
    t, k, p, rp = 0.8, 20, 0.9, 1.3
    toks, logits = eng.generate_batch(prompts, n, return_logits=True, temperature=t, top_k=k, top_p=p,
                                      repetition_penalty=rp, uniforms=uni)
    compared = 0
    for b in range(B):
        seen = list(prompts[b])
        for s_ in range(n):
            want, margin = R.sample_token(logits[b, s_], seen[-60:], t, k, p, rp, float(uni[b, s_]), detail=True)
            if margin >= 1e-4:
                compared += 1
                assert toks[b, s_] == want, (b, s_, toks[b, s_], want)
            seen.append(int(toks[b, s_]))
    assert compared >= B * n * 3 // 4


def test_embedding_and_rmsnorm_methods(dev):
    """get_embedding, rmsnorm and rmsnorm_inplace (cpu/mod.rs:285-347)
    against the oracle's rmsnorm_core restatement."""
    from oracle import retention_ref as R

    L, d, H, f, V = 1, 256, 2, 64, 30
    layers, emb = _model(L, d, f, V, 6, False)
    eng = _engine(layers, emb, H, 1, "float32", 1e-5)
    assert np.array_equal(eng.get_embedding(7), emb[7])
    with pytest.raises(ValueError):
        eng.get_embedding(V)
    rng = np.random.default_rng(1)
    x = rng.standard_normal(d).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    ref = R.rmsnorm_core(x, w, 1e-5)
    assert rel_err(eng.rmsnorm(x, w), ref) < 1e-5
    assert rel_err(eng.rmsnorm(x, w, eps=1e-2), R.rmsnorm_core(x, w, 1e-2)) < 1e-5
    y = x.copy()
    eng.rmsnorm_inplace(y, w)
    assert rel_err(y, ref) < 1e-5
    with pytest.raises(ValueError):
        eng.rmsnorm(x, w[:10])


def test_state_save_restore(dev, tmp_path):
    """The retention state saved mid-generation (to a host array and to an
    MTF file) and restored gives the same continuation."""
    L, d, H, f, V, B = 2, 256, 2, 64, 60, 2
    layers, emb = _model(L, d, f, V, 12, False)
    eng = _engine(layers, emb, H, B, "float32", 1e-5)
    prompts = np.array([[3, 9, 4], [7, 1, 8]], np.int32)
    eng.generate_batch(prompts, 3)
    snap = eng.get_state()
    p = str(tmp_path / "state.mtf")
    eng.save_state(p)
    want = eng.generate_batch(prompts, 4)
    eng.reset_memory()
    assert not eng.get_state().any()
    eng.set_state(snap)
    assert np.array_equal(eng.generate_batch(prompts, 4), want)
    eng.reset_memory()
    eng.load_state(p)
    assert np.array_equal(eng.get_state(), snap)
    assert np.array_equal(eng.generate_batch(prompts, 4), want)
    with pytest.raises(ValueError):
        eng.set_state(snap[:1])


def test_engine_validation(dev):
    from aceflow_b200.engine import AceEngine

    with pytest.raises(ValueError):
        AceEngine(1, 10, 3)
    eng = AceEngine(1, 64, 1)
    with pytest.raises(ValueError):
        eng.load_layer_weights(0, np.zeros(10), np.zeros(64 * 64), np.zeros(2 * 64 * 64), np.zeros(64 * 64),
                               np.ones(64), np.ones(64))
    with pytest.raises(ValueError):
        eng.forward_layer(0, np.zeros(64, np.float32))  # weights not loaded


@pytest.mark.parametrize("d", [1024, 2048, 4096, 8192, 512, 3000])
@pytest.mark.parametrize("with_w", [True, False])
def test_rmsnorm_to_bf16(dev, d, with_w):
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(d)
    x = torch.randn(5, d, generator=g, device=dev) * 3
    w = (1 + 0.1 * torch.randn(d, generator=g, device=dev)) if with_w else None
    y = cuda_ops.rms_norm_to_bf16(x, w, 1e-6)
    xd = x.double()
    ref = xd / torch.sqrt((xd * xd).mean(-1, keepdim=True) + 1e-6) * w.double() if with_w else xd
    assert rel_err(y.float().cpu().numpy(), ref.cpu().numpy()) < 8e-3


def test_engine_retention_step_packed_and_prefill_recurrent(dev):
    """AceEngine.retention_step / retention_step_packed / prefill_recurrent
    (aceflow-core/src/cpu/mod.rs:486-587) against the oracle's
    retention_step_core on the same per-layer state slice: the step's output,
    the packed split q | k | v, prefill_recurrent returning only the last
    token's output, the state left behind, and the reference's length and
    layer-index errors."""
    from aceflow_b200.engine import AceEngine

    L, d, H = 2, 512, 2
    dh = d // H
    gamma = np.array([1 - 2.0 ** (-5 - h) for h in range(H)], np.float32)
    rng = np.random.default_rng(17)
    eng = AceEngine(L, d, H, batch=1)
    states = np.zeros((L, H, dh, dh), np.float32)  # the reference's one-stream layout
    # retention_step on layer 1 (1-D vectors, as the reference takes them)
    q, k, v = (rng.standard_normal(d).astype(np.float32) for _ in range(3))
    ref = cpu_ref.retention_step_core(states, gamma, 1, H, dh, q, k, v)
    assert rel_err(eng.retention_step(1, q, k, v), ref) < 1e-5
    # retention_step_packed continues the same state
    qkv = rng.standard_normal(3 * d).astype(np.float32)
    ref = cpu_ref.retention_step_core(states, gamma, 1, H, dh, qkv[:d].copy(), qkv[d:2 * d].copy(), qkv[2 * d:].copy())
    got = eng.retention_step_packed(1, qkv)
    assert got.shape == (d,) and rel_err(got, ref) < 1e-5
    with pytest.raises(ValueError, match="Expected packed QKV vector of length"):
        eng.retention_step_packed(1, qkv[:-1])
    with pytest.raises(ValueError, match="Expected input vectors of length"):
        eng.retention_step(0, q[:-1], k, v)
    with pytest.raises(ValueError, match="out of range"):
        eng.retention_step(2, q, k, v)
    # prefill_recurrent on layer 0: flat [T*d] sequences, only the last output comes back
    T = 37
    qs, ks, vs = (rng.standard_normal(T * d).astype(np.float32) for _ in range(3))
    for t in range(T):
        last = cpu_ref.retention_step_core(states, gamma, 0, H, dh, qs[t * d:(t + 1) * d].copy(),
                                           ks[t * d:(t + 1) * d].copy(), vs[t * d:(t + 1) * d].copy())
    got = eng.prefill_recurrent(0, T, qs, ks, vs)
    assert got.shape == (d,) and rel_err(got, last) < 1e-4
    assert rel_err(eng.get_state()[:, 0], states) < 1e-5  # both layers' slices, layer 1 untouched by the prefill
    with pytest.raises(ValueError, match="Expected sequence vectors of length"):
        eng.prefill_recurrent(0, T, qs[:-d], ks, vs)
    with pytest.raises(ValueError, match="out of range"):
        eng.prefill_recurrent(5, T, qs, ks, vs)


def test_engine_retention_step_batched_streams(dev):
    """The batched engine (one state slice per stream) equals one oracle
    state per stream."""
    from aceflow_b200.engine import AceEngine

    L, d, H, B = 1, 256, 4, 3
    dh = d // H
    gamma = np.array([1 - 2.0 ** (-5 - h) for h in range(H)], np.float32)
    rng = np.random.default_rng(23)
    eng = AceEngine(L, d, H, batch=B)
    states = np.zeros((B, L, H, dh, dh), np.float32)
    for _ in range(3):
        q, k, v = (rng.standard_normal((B, d)).astype(np.float32) for _ in range(3))
        ref = np.stack([cpu_ref.retention_step_core(states[b], gamma, 0, H, dh, q[b].copy(), k[b].copy(), v[b].copy())
                        for b in range(B)])
        assert rel_err(eng.retention_step(0, q, k, v), ref) < 1e-5
    T = 9
    qs, ks, vs = (rng.standard_normal((B, T * d)).astype(np.float32) for _ in range(3))
    last = np.zeros((B, d), np.float32)
    for b in range(B):
        for t in range(T):
            sl = slice(t * d, (t + 1) * d)
            last[b] = cpu_ref.retention_step_core(states[b], gamma, 0, H, dh, qs[b, sl].copy(), ks[b, sl].copy(),
                                                  vs[b, sl].copy())
    got = eng.prefill_recurrent(0, T, qs, ks, vs)
    assert got.shape == (B, d) and rel_err(got, last) < 1e-4
    assert rel_err(eng.get_state()[0], states[:, 0]) < 1e-5
