"""Host-side API tests (no GPU): the mirrored reference API on CPU tensors,
device/dtype plumbing and argument validation."""
import numpy as np
import pytest

import aceflow_b200 as af
from conftest import golden, rel_err


def test_device_parsing():
    assert af.Device("cuda:3").type == "cuda" and af.Device("cuda:3").index == 3
    assert af.Device.cuda(1) == "cuda:1"
    assert af.Device.cpu() == "cpu"
    assert af.Device(None).type == "cpu"
    assert str(af.Device.cuda(2)) == "cuda:2"
    with pytest.raises(ValueError):
        af.Device("wgpu:0")
    with pytest.raises(ValueError):
        af.Device("tpu")


def test_tensor_basics():
    t = af.Tensor.zeros([2, 4])
    assert t.shape == [2, 4]
    assert np.allclose(t.numpy(), 0)
    u = af.Tensor(np.ones((2, 4)))
    assert (t + u).numpy().sum() == 8
    p = af.nn.Parameter(af.Tensor([1.0, 2.0]))
    assert p.numpy().tolist() == [1.0, 2.0]  # kept on every device (reference loses it without _native)
    with pytest.raises(ValueError):
        af.Tensor([1.0], dtype="bfloat16")  # bf16 is CUDA-only


def test_reference_shape_tests():
    # the reference's own test file, tests/test_framework.py:6-28 (shape tests)
    lin = af.nn.Linear(4, 8)
    assert lin(af.Tensor(np.ones((2, 4), np.float32))).shape == [2, 8]
    norm = af.nn.RMSNorm(8)
    assert norm(af.Tensor(np.random.randn(2, 8).astype(np.float32))).shape == [2, 8]
    ret = af.nn.MultiScaleRetention(d_model=64, num_heads=4)
    assert ret(af.Tensor(np.random.randn(2, 8, 64).astype(np.float32))).shape == [2, 8, 64]


@pytest.mark.parametrize("name", ["msr_config1.npz", "msr_small.npz"])
def test_msr_seeded_init_and_cpu_forward_match_reference(name):
    g = golden(name)
    B, T, d = g["x"].shape
    H = int(g["num_heads"])
    np.random.seed(0 if name == "msr_config1.npz" else 1)
    m = af.nn.MultiScaleRetention(d, H)
    for n in ("w_q", "w_k", "w_v", "w_o"):
        assert np.array_equal(getattr(m, n).numpy(), g[n]), n  # same draws, same order
    x = np.random.randn(B, T, d).astype(np.float32)
    assert np.array_equal(x, g["x"])
    assert rel_err(m(af.Tensor(x)).numpy(), g["out"]) == 0.0


def test_msr_cpu_recurrent_and_chunkwise_match_parallel():
    g = golden("msr_config1.npz")
    np.random.seed(0)
    m = af.nn.MultiScaleRetention(64, 4)
    out, state = m.forward_chunkwise(af.Tensor(g["x"]))
    assert rel_err(out.numpy(), g["out"]) < 1e-5
    assert state.shape == [2, 4, 16, 16]


def test_layers_cpu_match_reference():
    g = golden("layers_small.npz")
    x = af.Tensor(g["x"])
    norm = af.nn.RMSNorm(48)
    assert rel_err(norm(x).numpy(), g["rmsnorm_out"]) < 1e-7
    assert rel_err(af.ops.rms_norm(x, af.Tensor(g["ops_rms_norm_w"])).numpy(), g["ops_rms_norm_out"]) < 1e-7
    assert rel_err(af.ops.swiglu(x, af.Tensor(g["w_gate"]), af.Tensor(g["w_up"]), af.Tensor(g["w_down"])).numpy(),
                   g["swiglu_out"]) < 1e-6
    np.random.seed(2)
    af.nn.RMSNorm(48)
    ffn = af.nn.SwiGLU(48)
    lin = af.nn.Linear(48, 40)
    assert ffn.hidden_dim == 128
    assert np.array_equal(ffn.w_gate.weight.numpy(), g["w_gate"])
    assert np.array_equal(lin.weight.numpy(), g["lin_w"]) and np.array_equal(lin.bias.numpy(), g["lin_b"])
    assert rel_err(ffn(x).numpy(), g["swiglu_out"]) < 1e-6
    assert rel_err(lin(x).numpy(), g["linear_out"]) < 1e-6


def test_msr_rejects_bad_heads():
    with pytest.raises(ValueError):
        af.nn.MultiScaleRetention(10, 3)


def test_cuda_ops_reject_cpu_tensors():
    import torch

    from aceflow_b200 import cuda_ops

    with pytest.raises(ValueError):
        cuda_ops.rms_norm(torch.ones(2, 4), torch.ones(4), 1e-6)


def test_module_parameters_and_to_cpu():
    m = af.nn.SwiGLU(16, hidden_dim=32)
    names = [n for n, _ in m.named_parameters()]
    assert names == ["w_gate.weight", "w_up.weight", "w_down.weight"]
    m.to("cpu")
    assert all(p.device == "cpu" for p in m.parameters())


def test_noalloc_wrapper_rejects_bad_shapes_before_any_launch():
    """The allocation-free entry point cannot check sizes itself, so its
    wrapper rejects a mis-shaped state or weight (ValueError) before the
    call; CPU tensors reach the shape checks first."""
    import torch

    from aceflow_b200 import cuda_ops

    B, d, H = 2, 64, 4
    x = torch.zeros(B, d)
    gamma, rw = torch.ones(H), torch.ones(d)
    w_qkv, w_o = torch.zeros(3 * d, d), torch.zeros(d, d)
    with pytest.raises(ValueError, match="state shape"):
        cuda_ops.msr_decode_step_noalloc(x, torch.zeros(B, H, 8, 8), gamma, w_qkv, w_o, rw, 1e-6)
    state = torch.zeros(B, H, d // H, d // H)
    with pytest.raises(ValueError, match="w_qkv"):
        cuda_ops.msr_decode_step_noalloc(x, state, gamma, torch.zeros(2 * d, d), w_o, rw, 1e-6)
    with pytest.raises(ValueError, match="w_qkv"):
        cuda_ops.msr_decode_step_noalloc(x, state, gamma, w_qkv, torch.zeros(d, 2 * d), rw, 1e-6)
    with pytest.raises(ValueError, match="gamma"):
        cuda_ops.msr_decode_step_noalloc(x, state, torch.ones(H + 1), w_qkv, w_o, rw, 1e-6)
    with pytest.raises(ValueError, match="out"):
        cuda_ops.msr_decode_step_noalloc(x, state, gamma, w_qkv, w_o, rw, 1e-6, out=torch.zeros(B, d + 1))
    with pytest.raises(ValueError, match="CUDA"):  # well-shaped CPU tensors: the device check
        cuda_ops.msr_decode_step_noalloc(x, state, gamma, w_qkv, w_o, rw, 1e-6)


def test_gated_module_cpu_matches_float64_restatement():
    """gated=True (RetNet's gate and group norm, no reference counterpart):
    the CPU parallel and recurrent forms equal the oracle's float64
    restatement, and the reference's four weights are drawn unchanged."""
    from oracle import retention_ref as R

    np.random.seed(3)
    m = af.nn.MultiScaleRetention(64, 4, gated=True)
    m.group_norm_weight = af.nn.Parameter(af.Tensor(np.linspace(0.5, 1.5, 64).astype(np.float32)))
    m.group_norm_bias = af.nn.Parameter(af.Tensor(np.linspace(-0.1, 0.1, 64).astype(np.float32)))
    x = np.random.randn(2, 10, 64).astype(np.float32)
    f = lambda p: p.numpy().astype(np.float64)  # noqa: E731
    ref, _ = R.msr_gated_forward64(x, f(m.w_q), f(m.w_k), f(m.w_v), f(m.w_g), f(m.w_o), 4,
                                   f(m.group_norm_weight), f(m.group_norm_bias), 1e-6)
    assert rel_err(m(af.Tensor(x)).numpy(), ref) < 1e-5
    st = m.init_state(2)
    outs = []
    for t in range(10):
        o, st = m.forward_recurrent(af.Tensor(x[:, t]), st)
        outs.append(o.numpy())
    assert rel_err(np.stack(outs, 1), ref) < 1e-5
    np.random.seed(3)
    plain = af.nn.MultiScaleRetention(64, 4)
    for n in ("w_q", "w_k", "w_v", "w_o"):
        assert np.array_equal(getattr(m, n).numpy(), getattr(plain, n).numpy())
