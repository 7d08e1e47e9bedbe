"""The opt-in gated layer (RetNet's swish gate and per-head GroupNorm, Sun et
al. 2023; the reference has neither) on the GPU, against the oracle's
float64 restatement (oracle/retention_ref.py: group_norm_gate64,
msr_gated_forward64): the fused group-norm/gate kernel in every dtype
combination, the fp32 decode step (1e-4), the exact fp32 prefill (1e-4) and
the bf16 tensor-core prefill (2e-2), through af.nn.MultiScaleRetention."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import retention_ref as R

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.mark.parametrize("o_bf16,g_bf16,y_bf16", [(0, 0, 0), (1, 1, 1), (1, 0, 0), (0, 1, 1)])
@pytest.mark.parametrize("d,H", [(512, 2), (1024, 16), (96, 3)])
def test_group_norm_gate_kernel(dev, o_bf16, g_bf16, y_bf16, d, H):
    from aceflow_b200 import cuda_ops

    rows = 37
    g0 = torch.Generator(device=dev).manual_seed(d + H)
    o = 3 * torch.randn(rows, d, generator=g0, device=dev) + 0.5
    g = torch.randn(rows, d, generator=g0, device=dev)
    w = 1 + 0.1 * torch.randn(d, generator=g0, device=dev)
    b = 0.1 * torch.randn(d, generator=g0, device=dev)
    o = o.bfloat16() if o_bf16 else o
    g = g.bfloat16() if g_bf16 else g
    y = cuda_ops.group_norm_gate(o, g, H, w, b, 1e-6, out_dtype=torch.bfloat16 if y_bf16 else torch.float32)
    ref = R.group_norm_gate64(o.double().cpu().numpy(), g.double().cpu().numpy(), H, w.cpu().numpy(),
                              b.cpu().numpy(), 1e-6)
    tol = 1e-2 if y_bf16 else 1e-5
    assert rel_err(y.float().cpu().numpy(), ref) < tol


def _gated_module(d, H, seed):
    import aceflow_b200 as af

    rng = np.random.default_rng(seed)
    m = af.nn.MultiScaleRetention(d, H, gated=True)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).bfloat16().float().numpy()  # noqa: E731
    for n in ("w_q", "w_k", "w_v", "w_g", "w_o"):
        setattr(m, n, af.nn.Parameter(af.Tensor(bf(0.02 * rng.standard_normal((d, d))))))
    m.group_norm_weight = af.nn.Parameter(af.Tensor((1 + 0.1 * rng.standard_normal(d)).astype(np.float32)))
    m.group_norm_bias = af.nn.Parameter(af.Tensor((0.05 * rng.standard_normal(d)).astype(np.float32)))
    return m


def _ref(m, x):
    f = lambda p: p.numpy().astype(np.float64)  # noqa: E731
    return R.msr_gated_forward64(x, f(m.w_q), f(m.w_k), f(m.w_v), f(m.w_g), f(m.w_o), m.num_heads,
                                 f(m.group_norm_weight), f(m.group_norm_bias), 1e-6)[0]


def test_gated_module_decode_and_exact_prefill(dev):
    import aceflow_b200 as af

    B, T, d, H = 2, 20, 256, 2
    m = _gated_module(d, H, 81).to("cuda:0")
    x = np.random.default_rng(82).standard_normal((B, T, d)).astype(np.float32)
    ref = _ref(m, x)
    out = m(af.Tensor(x, device="cuda:0"))
    assert out.dtype == "float32" and rel_err(out.numpy(), ref) < 1e-4
    st = m.init_state(B)
    outs = []
    for t in range(T):
        o, st = m.forward_recurrent(af.Tensor(x[:, t], device="cuda:0"), st)
        outs.append(o.numpy())
    assert rel_err(np.stack(outs, 1), ref) < 1e-4


@pytest.mark.parametrize("chunk", [64, 128])
def test_gated_module_tensor_core_prefill(dev, chunk):
    import aceflow_b200 as af
    from aceflow_b200 import _lib

    B, T, d, H = 2, 300, 512, 2
    m = _gated_module(d, H, 83).to("cuda:0")
    xb = torch.from_numpy(np.random.default_rng(84).standard_normal((B, T, d)).astype(np.float32)).bfloat16()
    ref = _ref(m, xb.double().numpy())
    out, st = m.forward_chunkwise(af.Tensor(xb.to(dev), device="cuda:0", dtype="bfloat16"), chunk=chunk)
    torch.cuda.synchronize()
    assert _lib.check_device(0) == 0
    assert out.dtype == "bfloat16" and rel_err(out.numpy(), ref) < 2e-2
