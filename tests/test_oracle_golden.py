"""Pin the CPU oracle before trusting it.

Known-answer tests are the values in the reference's own Rust unit tests
(cited per test); fixtures come from running the reference's unmodified
Python modules (tests/golden/make_golden.py).  No GPU needed.
"""
import numpy as np
import pytest

from conftest import golden, rel_err
from oracle import cpu_ref
from oracle import retention_ref as R


# ---- known-answer tests from the reference's Rust sources -------------------
def test_kat_retention_step_numpy():
    # aceflow-core/src/cpu/recurrence.rs:49-65
    state = np.zeros((1, 2, 2), np.float32)
    out = R.retention_step_core(state, np.array([0.5], np.float32),
                                np.array([2, 3], np.float32), np.array([4, 5], np.float32),
                                np.array([6, 7], np.float32))
    assert state.reshape(-1).tolist() == [24.0, 28.0, 30.0, 35.0]
    assert out.tolist() == [138.0, 161.0]


def test_kat_retention_step_c():
    state = np.zeros(4, np.float32)
    out = cpu_ref.retention_step_core(state, np.array([0.5], np.float32), 0, 1, 2,
                                      np.array([2, 3], np.float32), np.array([4, 5], np.float32),
                                      np.array([6, 7], np.float32))
    assert state.tolist() == [24.0, 28.0, 30.0, 35.0]
    assert out.tolist() == [138.0, 161.0]


def test_kat_rmsnorm():
    # aceflow-core/src/cpu/norm.rs:85-93
    x = np.array([1, 2, 3, 4], np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(7.5) + np.float32(1e-5))
    for y in (R.rmsnorm_core(x, np.ones(4, np.float32), 1e-5),
              cpu_ref.rmsnorm_core(x, np.ones(4, np.float32), 1e-5)):
        assert np.all(np.abs(y - x * inv) < 1e-6)


def test_kat_swiglu():
    # aceflow-core/src/cpu/swiglu.rs:25-29 (zero gate) and nn/mod.rs:51-57 (packed split)
    assert R.swiglu_packed(np.array([0.0, 4.0], np.float32), 1).tolist() == [0.0]
    assert cpu_ref.swiglu_forward(np.array([0.0, 4.0], np.float32), 1).tolist() == [0.0]
    out = R.swiglu_packed(np.array([[0.0, 1.0, 2.0, 3.0]], np.float32), 2)
    assert out[0, 0] == 0.0
    assert abs(out[0, 1] - 3.0 / (1.0 + np.exp(-1.0))) < 1e-6


def test_kat_gemv_simd_matches_scalar():
    # aceflow-core/src/cpu/gemv.rs:320-331
    w = (np.arange(40, dtype=np.float32) * np.float32(0.125) - np.float32(2.0)).reshape(4, 10)
    x = np.arange(10, dtype=np.float32) * np.float32(0.25)
    expected = cpu_ref.gemv(w, x, scalar=True)
    actual = cpu_ref.gemv(w, x)
    assert np.all(np.abs(expected - actual) < 1e-4)
    assert np.all(np.abs(R.gemv_scalar(w, x) - expected) < 1e-6)


def test_kat_dot():
    # aceflow-core/src/cpu/gemv.rs:333-348 (dot on 17 elements)
    a = np.arange(17, dtype=np.float32) * np.float32(0.5) - np.float32(2.0)
    b = np.arange(17, dtype=np.float32) * np.float32(0.25)
    ref = float(np.sum(a.astype(np.float64) * b))
    assert abs(cpu_ref.lib().oref_dot_product(cpu_ref._p(a), cpu_ref._p(b), 17) - ref) < 1e-4


def test_kat_sampler_restatement():
    """The full sampler restatement against the reference's tests
    (sampler.rs:187-197) and hand-worked cases of sampler.rs:130-179."""
    assert R.sample_token([1.0, 3.0, 2.0], [], 0.0, 0, 1.0, 1.0) == 1
    assert R.sample_token([1.0, 3.0, 2.0], [1], 0.0, 0, 1.0, 10.0) == 2
    # logits ln 1, ln 2, ln 3, ln 4 at temperature 1: probabilities .1 .2 .3 .4
    lg = np.log(np.array([1.0, 2.0, 3.0, 4.0], np.float32))
    # sorted 3, 2, 1, 0 with running sums .4 .7 .9 1.0
    assert [R.sample_token(lg, (), 1.0, 0, 1.0, 1.0, u) for u in (0.0, 0.39, 0.41, 0.69, 0.71, 0.89, 0.91)] == \
        [3, 3, 2, 2, 1, 1, 0]
    # top_k 2 keeps 3, 2 (renormalised 4/7, 3/7); top_p 0.5 keeps 3, 2 (.7 is the first sum > .5),
    # top_p 0.3 keeps only 3
    assert R.sample_token(lg, (), 1.0, 2, 1.0, 1.0, 0.56) == 3
    assert R.sample_token(lg, (), 1.0, 2, 1.0, 1.0, 0.58) == 2
    assert R.sample_token(lg, (), 1.0, 0, 0.5, 1.0, 0.99) == 2
    assert R.sample_token(lg, (), 1.0, 0, 0.3, 1.0, 0.99) == 3
    # penalty 2 on token 3 (once, though listed twice): ln4 / 2 = ln2, so 1 and 3
    # tie at ln 2; probabilities 3/8 (token 2), 2/8, 2/8, 1/8 with the tie in
    # index order: a draw at 0.5 lands on token 1, at 0.7 on token 3
    assert R.sample_token(lg, [3, 3], 1.0, 0, 1.0, 2.0, 0.5) == 1
    assert R.sample_token(lg, [3, 3], 1.0, 0, 1.0, 2.0, 0.7) == 3


def test_kat_greedy_sampler():
    # aceflow-core/src/cpu/sampler.rs:187-197
    assert R.greedy_token([1.0, 3.0, 2.0], [], 1.0) == 1
    assert R.greedy_token([1.0, 3.0, 2.0], [1], 10.0) == 2
    assert R.greedy_token([5.0, 5.0, 1.0]) == 0  # first maximum wins (sampler.rs:119-126)


def test_kat_linear_layout():
    # aceflow-core/src/nn/mod.rs:34-39: PyTorch (out, in) layout
    w = np.array([[1.0, 2.0], [-1.0, 3.0]], np.float32)
    b = np.array([0.5, -0.5], np.float32)
    assert R.linear_py(np.array([[2.0, 4.0]], np.float32), w, b).tolist() == [[10.5, 9.5]]


def test_kat_gemm_bt():
    # aceflow-core/src/tensor/mod.rs:577-582
    a = np.array([1, 2, 3, 4], np.float32).reshape(2, 2)
    b = np.array([2, 1, -1, 3], np.float32).reshape(2, 2)
    assert R.gemm_bt(a, b).reshape(-1).tolist() == [4.0, 5.0, 10.0, 9.0]


def test_gamma_formula():
    g = R.gammas(8)
    assert g.dtype == np.float32
    assert g.tolist() == [np.float32(1.0 - 2.0 ** (-5 - h)) for h in range(8)]


# ---- fixtures from the unmodified reference Python ---------------------------
@pytest.mark.parametrize("name", ["msr_config1.npz", "msr_small.npz"])
def test_parallel_form_matches_reference_fixture(name):
    g = golden(name)
    out = R.msr_parallel(g["x"], g["w_q"], g["w_k"], g["w_v"], g["w_o"], int(g["num_heads"]),
                         g["ret_norm_w"], float(g["eps"]))
    assert rel_err(out, g["out"]) < 1e-6


@pytest.mark.parametrize("name", ["msr_config1.npz", "msr_small.npz"])
def test_recurrent_restatement_matches_reference_fixture(name):
    """Token-serial recurrence (recurrence.rs) equals the reference's parallel
    form (retention.py) on the reference's own output."""
    g = golden(name)
    x = g["x"]
    B, T, d = x.shape
    H = int(g["num_heads"])
    state = np.zeros((B, H, d // H, d // H), np.float32)
    w_qkv = np.concatenate([g["w_q"], g["w_k"], g["w_v"]], 0)
    out = np.stack([R.msr_recurrent_step(x[:, t], state, R.gammas(H), w_qkv, g["w_o"], g["ret_norm_w"],
                                         float(g["eps"])) for t in range(T)], 1)
    assert rel_err(out, g["out"]) < 1e-5


@pytest.mark.parametrize("name", ["msr_config1.npz", "msr_small.npz"])
def test_c_restatement_matches_reference_fixture(name):
    g = golden(name)
    x = np.ascontiguousarray(g["x"])
    B, T, d = x.shape
    H = int(g["num_heads"])
    state = np.zeros((B, H, d // H, d // H), np.float32)
    w_qkv = np.ascontiguousarray(np.concatenate([g["w_q"], g["w_k"], g["w_v"]], 0))
    out = cpu_ref.msr_prefill_recurrent(x, state, R.gammas(H), w_qkv, np.ascontiguousarray(g["w_o"]),
                                        np.ascontiguousarray(g["ret_norm_w"]), float(g["eps"]))
    assert rel_err(out, g["out"]) < 1e-5


@pytest.mark.parametrize("chunk", [1, 3, 4, 16, 64])
def test_chunkwise_form_matches_reference_fixture(chunk):
    g = golden("msr_small.npz")
    x = g["x"].astype(np.float64)
    B, T, d = x.shape
    H = int(g["num_heads"])
    hd = d // H
    q = (x @ g["w_q"].T).reshape(B, T, H, hd).transpose(0, 2, 1, 3)
    k = (x @ g["w_k"].T).reshape(B, T, H, hd).transpose(0, 2, 1, 3)
    v = (x @ g["w_v"].T).reshape(B, T, H, hd).transpose(0, 2, 1, 3)
    par = R.retention_parallel_core64(q, k, v, R.gammas(H))
    chk, _ = R.retention_chunkwise64(q, k, v, R.gammas(H), chunk)
    assert rel_err(chk, par) < 1e-12
    full = R.msr_forward64(g["x"], g["w_q"], g["w_k"], g["w_v"], g["w_o"], H, g["ret_norm_w"], float(g["eps"]))
    assert rel_err(full, g["out"]) < 1e-5


def test_layers_match_reference_fixture():
    g = golden("layers_small.npz")
    x = g["x"]
    assert rel_err(R.rms_norm_py(x, np.ones(48, np.float32), float(g["rmsnorm_eps"])), g["rmsnorm_out"]) < 1e-7
    assert rel_err(R.rms_norm_py(x, g["ops_rms_norm_w"], 1e-6), g["ops_rms_norm_out"]) < 1e-7
    assert rel_err(R.swiglu_py(x, g["w_gate"], g["w_up"], g["w_down"]), g["swiglu_out"]) < 1e-6
    assert rel_err(R.linear_py(x, g["lin_w"], g["lin_b"]), g["linear_out"]) < 1e-6


def test_decoder_layer_c_matches_float64():
    rng = np.random.default_rng(3)
    B, d, H, f = 3, 32, 2, 48
    layer = dict(
        w_qkv=(rng.standard_normal((3 * d, d)) * 0.1).astype(np.float32),
        w_o=(rng.standard_normal((d, d)) * 0.1).astype(np.float32),
        w_gate_up=(rng.standard_normal((2 * f, d)) * 0.1).astype(np.float32),
        w_down=(rng.standard_normal((d, f)) * 0.1).astype(np.float32),
        norm1=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
        norm2=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
        ret_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
    )
    x = rng.standard_normal((B, d)).astype(np.float32)
    states = np.zeros((B, 1, H, d // H, d // H), np.float32)
    st64 = np.zeros((B, H, d // H, d // H))
    x64 = x.astype(np.float64)
    xc = x.copy()
    for _ in range(5):
        cpu_ref.forward_layer(xc, [layer], 0, states, R.gammas(H), 1e-5)
        x64 = R.decoder_layer64(x64, layer, st64, R.gammas(H), 1e-5)
    assert rel_err(xc, x64) < 1e-5
