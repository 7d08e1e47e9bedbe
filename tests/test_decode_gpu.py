"""GPU parity of the fp32 decode path against the CPU oracle.

Every call goes through libaceflow_cuda.so's C ABI (via aceflow_b200's
ctypes binding).  Tolerance for fp32 paths: max|y - y_ref| / max|y_ref| <= 1e-4
(the bar for fp32 retention); most cases land near 1e-6.
"""
import numpy as np
import pytest
import torch

from conftest import golden, rel_err
from oracle import cpu_ref
from oracle import retention_ref as R

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_kat_retention_step(dev):
    """aceflow-core/src/cpu/recurrence.rs:49-65 on the GPU (head_dim 2)."""
    from aceflow_b200 import cuda_ops

    state = torch.zeros(1, 1, 2, 2, device=dev)
    out = cuda_ops.retention_step(state, T(np.array([0.5], np.float32), dev), T(np.array([[2, 3]], np.float32), dev),
                                  T(np.array([[4, 5]], np.float32), dev), T(np.array([[6, 7]], np.float32), dev))
    assert state.flatten().tolist() == [24.0, 28.0, 30.0, 35.0]
    assert out.flatten().tolist() == [138.0, 161.0]


@pytest.mark.parametrize("dh", [2, 4, 6, 16, 32, 48, 64, 128, 256])
def test_retention_step_matches_oracle(dev, dh):
    from aceflow_b200 import cuda_ops

    rng = np.random.default_rng(dh)
    B, H = 3, 2
    d = H * dh
    gamma = R.gammas(H)
    st = np.zeros((B, H, dh, dh), np.float32)
    st_d = torch.zeros(B, H, dh, dh, device=dev)
    for step in range(3):
        qkv = rng.standard_normal((B, 3 * d)).astype(np.float32)
        outs = []
        for b in range(B):
            flat = st[b].reshape(-1)
            outs.append(cpu_ref.retention_step_core(flat, gamma, 0, H, dh, qkv[b, :d].copy(), qkv[b, d:2 * d].copy(),
                                                    qkv[b, 2 * d:].copy()))
            st[b] = flat.reshape(H, dh, dh)
        ref = np.stack(outs)
        q = T(qkv, dev)
        out = cuda_ops.retention_step(st_d, T(gamma, dev), q[:, :d], q[:, d:2 * d], q[:, 2 * d:])
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), ref) < 1e-5, step
        assert rel_err(st_d.cpu().numpy(), st) < 1e-5, step


@pytest.mark.parametrize("dh", [6, 16, 64, 128, 256])
def test_retention_scan_matches_oracle(dev, dh):
    from aceflow_b200 import cuda_ops

    rng = np.random.default_rng(100 + dh)
    B, H, Tn = 2, 2, 7
    d = H * dh
    gamma = R.gammas(H)
    qkv = rng.standard_normal((B, Tn, 3 * d)).astype(np.float32)
    st = np.zeros((B, H, dh, dh), np.float32)
    ref = np.zeros((B, Tn, d), np.float32)
    for b in range(B):
        flat = st[b].reshape(-1)
        for t in range(Tn):
            ref[b, t] = cpu_ref.retention_step_core(flat, gamma, 0, H, dh, qkv[b, t, :d].copy(),
                                                    qkv[b, t, d:2 * d].copy(), qkv[b, t, 2 * d:].copy())
        st[b] = flat.reshape(H, dh, dh)
    st_d = torch.zeros(B, H, dh, dh, device=dev)
    q = T(qkv, dev)
    out = cuda_ops.retention_scan(st_d, T(gamma, dev), q[..., :d], q[..., d:2 * d], q[..., 2 * d:])
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), ref) < 1e-5
    assert rel_err(st_d.cpu().numpy(), st) < 1e-5


@pytest.mark.parametrize("rows,d", [(1, 4), (5, 48), (3, 2048), (7, 1001)])
def test_rmsnorm_matches_oracle(dev, rows, d):
    from aceflow_b200 import cuda_ops

    rng = np.random.default_rng(rows * d)
    x = rng.standard_normal((rows, d)).astype(np.float32)
    r = rng.standard_normal((rows, d)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    for eps in (1e-5, 1e-6):
        ref = np.stack([cpu_ref.rmsnorm_core(x[i], w, eps) for i in range(rows)])
        y = cuda_ops.rms_norm(T(x, dev), T(w, dev), eps)
        assert rel_err(y.cpu().numpy(), ref) < 1e-6
    s = torch.empty(rows, d, device=dev)
    y = cuda_ops.rms_norm(T(x, dev), T(w, dev), 1e-5, residual=T(r, dev), sum_out=s)
    ref = np.stack([cpu_ref.rmsnorm_core(x[i] + r[i], w, 1e-5) for i in range(rows)])
    assert rel_err(y.cpu().numpy(), ref) < 1e-6
    assert rel_err(s.cpu().numpy(), x + r) == 0.0
    yb = cuda_ops.rms_norm(T(x, dev).bfloat16(), T(w, dev), 1e-6)
    assert rel_err(yb.float().cpu().numpy(), R.rms_norm_py(x, w, 1e-6)) < 2e-2


def test_swiglu_and_silu_match_oracle(dev):
    from aceflow_b200 import cuda_ops

    rng = np.random.default_rng(7)
    gu = (3 * rng.standard_normal((5, 2 * 37))).astype(np.float32)
    ref = np.stack([cpu_ref.swiglu_forward(gu[i], 37) for i in range(5)])
    assert rel_err(cuda_ops.swiglu_packed(T(gu, dev)).cpu().numpy(), ref) < 1e-6
    g = gu[:, :37].copy()
    assert rel_err(cuda_ops.silu_mul(T(g, dev)).cpu().numpy(), R.silu(g)) < 1e-6
    assert cuda_ops.swiglu_packed(T(np.array([[0.0, 4.0]], np.float32), dev)).item() == 0.0  # swiglu.rs:25-29


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (5, 7, 13), (64, 64, 64), (256, 6144, 2048), (33, 2048, 5632)])
def test_linear_matches_float64(dev, M, N, K):
    from aceflow_b200 import cuda_ops

    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y = cuda_ops.linear(T(x, dev), T(w, dev), T(b, dev)).cpu().numpy()
    ref = x.astype(np.float64) @ w.T.astype(np.float64) + b
    assert rel_err(y, ref) < 1e-5


def test_linear_kat_layout(dev):
    # aceflow-core/src/nn/mod.rs:34-39
    from aceflow_b200 import cuda_ops

    y = cuda_ops.linear(T(np.array([[2.0, 4.0]], np.float32), dev), T(np.array([[1.0, 2.0], [-1.0, 3.0]], np.float32), dev),
                        T(np.array([0.5, -0.5], np.float32), dev))
    assert y.cpu().numpy().tolist() == [[10.5, 9.5]]


@pytest.mark.parametrize("B,d,H,steps", [(4, 256, 2, 4), (3, 2048, 8, 3), (2, 96, 4, 5)])
def test_msr_decode_step_matches_oracle(dev, B, d, H, steps):
    from aceflow_b200 import cuda_ops

    rng = np.random.default_rng(B * d + H)
    dh = d // H
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    gamma = R.gammas(H)
    st = np.zeros((B, H, dh, dh), np.float32)
    st_d = torch.zeros(B, H, dh, dh, device=dev)
    args = [T(a, dev) for a in (gamma, w_qkv, w_o, ret_w)]
    for s in range(steps):
        x = rng.standard_normal((B, d)).astype(np.float32)
        ref = cpu_ref.msr_decode_step(x, st, gamma, w_qkv, w_o, ret_w, 1e-6)
        out = cuda_ops.msr_decode_step(T(x, dev), st_d, *args, 1e-6)
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), ref) < TOL, s
        assert rel_err(st_d.cpu().numpy(), st) < TOL, s


def test_msr_decode_step_full_config(dev):
    """The decode workload's full shape (d=2048, 8 heads, 256 streams), two
    steps from a zero state, against the C restatement of the reference."""
    from aceflow_b200 import cuda_ops

    B, d, H = 256, 2048, 8
    rng = np.random.default_rng(2)
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = np.ones(d, np.float32)
    gamma = R.gammas(H)
    st = np.zeros((B, H, d // H, d // H), np.float32)
    st_d = torch.zeros(B, H, d // H, d // H, device=dev)
    args = [T(a, dev) for a in (gamma, w_qkv, w_o, ret_w)]
    for s in range(2):
        x = rng.standard_normal((B, d)).astype(np.float32)
        ref = cpu_ref.msr_decode_step(x, st, gamma, w_qkv, w_o, ret_w, 1e-6)
        out = cuda_ops.msr_decode_step(T(x, dev), st_d, *args, 1e-6)
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), ref) < TOL
    assert rel_err(st_d.cpu().numpy(), st) < TOL


def test_msr_decode_rejects_bad_shapes(dev):
    from aceflow_b200 import _lib

    with pytest.raises(ValueError):
        _lib.call("af_msr_decode_step_f32", _lib.context(0), 1, 1, 1, 1, 1, 1, 1e-6, 2, 10, 3, 1, None)


# ---- module level: the mirrored reference API on a CUDA device -------------
@pytest.mark.parametrize("name", ["msr_config1.npz", "msr_small.npz"])
def test_msr_module_cuda_matches_reference_fixture(dev, name):
    import aceflow_b200 as af

    g = golden(name)
    B, Tn, d = g["x"].shape
    np.random.seed(0 if name == "msr_config1.npz" else 1)
    m = af.nn.MultiScaleRetention(d, int(g["num_heads"])).to("cuda:0")
    x = af.Tensor(g["x"], device="cuda:0")
    assert rel_err(m(x).numpy(), g["out"]) < TOL
    # recurrent form, token by token, equals the reference's parallel form
    state = m.init_state(B)
    outs = []
    for t in range(Tn):
        o, state = m.forward_recurrent(af.Tensor(g["x"][:, t], device="cuda:0"), state)
        outs.append(o.numpy())
    assert rel_err(np.stack(outs, 1), g["out"]) < TOL


def test_layers_cuda_match_reference_fixture(dev):
    import aceflow_b200 as af

    g = golden("layers_small.npz")
    x = af.Tensor(g["x"], device="cuda:0")
    assert rel_err(af.nn.RMSNorm(48).to("cuda:0")(x).numpy(), g["rmsnorm_out"]) < 1e-6
    assert rel_err(af.ops.rms_norm(x, af.Tensor(g["ops_rms_norm_w"], "cuda:0")).numpy(), g["ops_rms_norm_out"]) < 1e-6
    assert rel_err(af.ops.swiglu(x, *(af.Tensor(g[n], "cuda:0") for n in ("w_gate", "w_up", "w_down"))).numpy(),
                   g["swiglu_out"]) < TOL
    np.random.seed(2)
    af.nn.RMSNorm(48)
    ffn = af.nn.SwiGLU(48).to("cuda:0")
    lin = af.nn.Linear(48, 40).to("cuda:0")
    assert rel_err(ffn(x).numpy(), g["swiglu_out"]) < TOL
    assert rel_err(lin(x).numpy(), g["linear_out"]) < TOL
    assert rel_err((x @ af.Tensor(g["lin_w"].T.copy(), "cuda:0") + af.Tensor(g["lin_b"], "cuda:0")).numpy(),
                   g["linear_out"]) < TOL


@pytest.mark.parametrize("B,d,H,groups", [(256, 2048, 8, "4"), (256, 2048, 8, "1"), (5, 512, 2, "2"), (130, 1024, 8, "8"),
                                           (130, 1024, 8, "1"), (100, 512, 4, "1"), (65, 256, 1, "1")])
def test_msr_decode_step_split_weights_matches_oracle(dev, B, d, H, groups):
    """Head-major, tf32-split weights give the fp32 decode step, sequential
    (1 head group) or pipelined over head groups on three streams."""
    from aceflow_b200 import _lib, cuda_ops

    _lib.set_option(0, "decode_head_groups", int(groups))

    rng = np.random.default_rng(B + d)
    dh = d // H
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    gamma = R.gammas(H)
    hi, lo = cuda_ops.split_tf32(T(w_qkv, dev))
    assert torch.equal(hi + lo, T(w_qkv, dev))
    assert torch.equal(hi, (hi.view(torch.int32) & ~0x1FFF).view(torch.float32))
    packed = cuda_ops.pack_qkv_heads(T(w_qkv, dev), H)
    ref_pack = w_qkv.reshape(3, H, dh, d).transpose(1, 0, 2, 3).reshape(3 * d, d)
    assert np.array_equal(packed.cpu().numpy(), ref_pack)
    wq_s, wo_s = cuda_ops.prepare_decode_weights(T(w_qkv, dev), T(w_o, dev), H)
    st = np.zeros((B, H, dh, dh), np.float32)
    st_d = torch.zeros(B, H, dh, dh, device=dev)
    for s in range(2):
        x = rng.standard_normal((B, d)).astype(np.float32)
        ref = cpu_ref.msr_decode_step(x, st, gamma, w_qkv, w_o, ret_w, 1e-6)
        out = cuda_ops.msr_decode_step_split(T(x, dev), st_d, T(gamma, dev), wq_s, wo_s, T(ret_w, dev), 1e-6)
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), ref) < TOL, s
        assert rel_err(st_d.cpu().numpy(), st) < TOL, s
    _lib.set_option(0, "decode_head_groups", 1)


@pytest.mark.parametrize("pairs", [0, 1])
def test_msr_decode_step_split_pairs_option(dev, pairs):
    """The transposed QKV projection on CTA pairs and on single CTAs give the
    same fp32 decode step (af_set_option "decode_pairs")."""
    from aceflow_b200 import _lib, cuda_ops

    B, d, H = 256, 1024, 4
    rng = np.random.default_rng(77)
    dh = d // H
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    gamma = R.gammas(H)
    wq_s, wo_s = cuda_ops.prepare_decode_weights(T(w_qkv, dev), T(w_o, dev), H)
    st = np.zeros((B, H, dh, dh), np.float32)
    st_d = torch.zeros(B, H, dh, dh, device=dev)
    _lib.set_option(0, "decode_pairs", pairs)
    try:
        for s in range(2):
            x = rng.standard_normal((B, d)).astype(np.float32)
            ref = cpu_ref.msr_decode_step(x, st, gamma, w_qkv, w_o, ret_w, 1e-6)
            out = cuda_ops.msr_decode_step_split(T(x, dev), st_d, T(gamma, dev), wq_s, wo_s, T(ret_w, dev), 1e-6)
            torch.cuda.synchronize()
            assert rel_err(out.cpu().numpy(), ref) < TOL, s
            assert rel_err(st_d.cpu().numpy(), st) < TOL, s
    finally:
        _lib.set_option(0, "decode_pairs", 1)
    assert _lib.check_device(0) == 0


@pytest.mark.parametrize("groups", [1, 4])
def test_msr_decode_step_split_four_producers(dev, groups):
    """Decode step with four TMA producer threads per GEMM CTA, sequential and
    over four head groups on three streams (the 3xTF32 GEMMs there have a
    3-stage ring, so the producer count is capped at 3): equal to the oracle."""
    from aceflow_b200 import _lib, cuda_ops

    B, d, H = 256, 2048, 8
    rng = np.random.default_rng(91)
    dh = d // H
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    ret_w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    gamma = R.gammas(H)
    wq_s, wo_s = cuda_ops.prepare_decode_weights(T(w_qkv, dev), T(w_o, dev), H)
    st = np.zeros((B, H, dh, dh), np.float32)
    st_d = torch.zeros(B, H, dh, dh, device=dev)
    _lib.set_option(0, "gemm_producers", 4)
    _lib.set_option(0, "decode_head_groups", groups)
    try:
        for s in range(2):
            x = rng.standard_normal((B, d)).astype(np.float32)
            ref = cpu_ref.msr_decode_step(x, st, gamma, w_qkv, w_o, ret_w, 1e-6)
            out = cuda_ops.msr_decode_step_split(T(x, dev), st_d, T(gamma, dev), wq_s, wo_s, T(ret_w, dev), 1e-6)
            torch.cuda.synchronize()
            assert rel_err(out.cpu().numpy(), ref) < TOL, s
            assert rel_err(st_d.cpu().numpy(), st) < TOL, s
    finally:
        _lib.set_option(0, "gemm_producers", 1)
        _lib.set_option(0, "decode_head_groups", 1)
    assert _lib.check_device(0) == 0
