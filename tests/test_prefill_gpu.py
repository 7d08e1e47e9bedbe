"""GPU parity of the tensor-core chunkwise prefill (bf16 operands, fp32
accumulation) against the float64 oracle.  Tolerance for the bf16 path:
max|y - y_ref| / max|y_ref| <= 2e-2."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import retention_ref as R

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _qkv(B, T, H, seed, dev, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    d = H * 256
    return (scale * torch.randn(B * T, 3 * d, generator=g, device=dev)).bfloat16()


def _core_ref(qkv, B, T, H, state0=None):
    d = H * 256
    a = qkv.float().cpu().numpy().astype(np.float64).reshape(B, T, 3, H, 256)
    q, k, v = (a[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    o, S = R.retention_chunkwise64(q, k, v, R.gammas(H), 64, state0)
    return o.transpose(0, 2, 1, 3).reshape(B * T, d), S


@pytest.mark.parametrize("chunk", [64, 128])
@pytest.mark.parametrize("B,T,H", [(1, 64, 1), (2, 100, 2), (1, 257, 2), (3, 200, 1), (1, 1000, 8), (2, 128, 1),
                                   (1, 129, 1), (1, 1, 1), (2, 3, 2)])
def test_chunkwise_core_matches_oracle(dev, B, T, H, chunk):
    from aceflow_b200 import _lib, cuda_ops

    qkv = _qkv(B, T, H, B * 1000 + T + H, dev, scale=0.5)
    gamma = cuda_ops.gammas(H, dev)
    w = (1 + 0.1 * torch.randn(H * 256, device=dev))
    out, ss, st = cuda_ops.retention_chunkwise_bf16(qkv, B, T, H, gamma, norm_w=w, chunk=chunk)
    torch.cuda.synchronize()
    assert _lib.check_device(0) == 0
    ref, S = _core_ref(qkv, B, T, H)
    wn = w.cpu().numpy().astype(np.float64)
    assert rel_err(out.float().cpu().numpy(), ref * wn) < TOL
    assert rel_err(st.cpu().numpy(), S) < TOL
    rs = ss.cpu().numpy().sum(1)
    assert rel_err(rs, (ref * ref).sum(1)) < TOL


@pytest.mark.parametrize("chunk", [64, 128])
def test_chunkwise_state_carry(dev, chunk):
    """Two calls chained through the state equal one call over the whole
    sequence (and a non-zero initial state is honoured)."""
    from aceflow_b200 import cuda_ops

    B, H, T1, T2 = 2, 2, 130, 70
    qkv = _qkv(B, T1 + T2, H, 7, dev, scale=0.5)
    gamma = cuda_ops.gammas(H, dev)
    full, _, S_full = cuda_ops.retention_chunkwise_bf16(qkv, B, T1 + T2, H, gamma, chunk=chunk)
    q3 = qkv.view(B, T1 + T2, -1)
    a = q3[:, :T1].contiguous().view(B * T1, -1)
    b = q3[:, T1:].contiguous().view(B * T2, -1)
    o1, _, S1 = cuda_ops.retention_chunkwise_bf16(a, B, T1, H, gamma, chunk=chunk)
    o2, _, S2 = cuda_ops.retention_chunkwise_bf16(b, B, T2, H, gamma, state_in=S1, chunk=chunk)
    f = full.float().view(B, T1 + T2, -1)
    assert rel_err(o1.float().view(B, T1, -1).cpu().numpy(), f[:, :T1].cpu().numpy()) < 1e-2
    assert rel_err(o2.float().view(B, T2, -1).cpu().numpy(), f[:, T1:].cpu().numpy()) < TOL
    assert rel_err(S2.cpu().numpy(), S_full.cpu().numpy()) < TOL


@pytest.mark.parametrize("chunk", [64, 128])
@pytest.mark.parametrize("B,T,H", [(2, 96, 2), (1, 300, 8)])
def test_msr_prefill_matches_float64(dev, B, T, H, chunk):
    from aceflow_b200 import _lib, cuda_ops

    d = H * 256
    rng = np.random.default_rng(B + T + H)
    x = rng.standard_normal((B, T, d)).astype(np.float32)
    wq, wk, wv, wo = ((0.02 * rng.standard_normal((d, d))).astype(np.float32) for _ in range(4))
    rw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    tb = lambda a: torch.from_numpy(a).to(dev).bfloat16()  # noqa: E731
    xb, wqkv, wob = tb(x), tb(np.concatenate([wq, wk, wv])), tb(wo)
    out, st = cuda_ops.msr_prefill_bf16(xb, wqkv, wob, torch.from_numpy(rw).to(dev), cuda_ops.gammas(H, dev), 1e-6,
                                        chunk=chunk)
    torch.cuda.synchronize()
    assert _lib.check_device(0) == 0
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    wq_, wk_, wv_ = np.split(f(wqkv), 3)
    ref = R.msr_forward64(f(xb), wq_, wk_, wv_, f(wob), H, rw, 1e-6)
    assert rel_err(out.cpu().numpy(), ref) < TOL
    # against the fp32 weights/inputs too (the bf16 quantisation is inside the tolerance)
    ref32 = R.msr_forward64(x, wq, wk, wv, wo, H, rw, 1e-6)
    assert rel_err(out.cpu().numpy(), ref32) < TOL


def test_prefill_then_decode_continues_the_state(dev):
    """Prefill T tokens, then one fp32 decode step from the returned state,
    equals the recurrence over T+1 tokens."""
    from aceflow_b200 import cuda_ops

    B, H, T = 2, 2, 77
    d = H * 256
    rng = np.random.default_rng(11)
    x = rng.standard_normal((B, T + 1, d)).astype(np.float32)
    w = [(0.02 * rng.standard_normal((d, d))).astype(np.float32) for _ in range(4)]
    w = [torch.from_numpy(a).to(dev).bfloat16().float() for a in w]  # bf16-representable weights
    xb = torch.from_numpy(x).to(dev).bfloat16()
    rw = torch.ones(d, device=dev)
    gamma = cuda_ops.gammas(H, dev)
    wqkv = torch.cat(w[:3]).contiguous()
    _, st = cuda_ops.msr_prefill_bf16(xb[:, :T].contiguous(), wqkv.bfloat16(), w[3].bfloat16(), rw, gamma, 1e-6)
    out = cuda_ops.msr_decode_step(xb[:, T].float().contiguous(), st, gamma, wqkv, w[3], rw, 1e-6)
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    ref = R.msr_forward64(f(xb), *(f(a) for a in w), H, None, 1e-6)[:, T]
    assert rel_err(out.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("chunk", [64, 128])
@pytest.mark.parametrize("nseg", [1, 3, 0])
def test_chunkwise_segments_match_single_pass(dev, nseg, chunk):
    """Sequence segments (state pass + scan + full pass) give the recurrence's
    result: forced 1 (single pass), 3 (ragged last segment) and auto."""
    from aceflow_b200 import _lib, cuda_ops

    B, T, H = 1, 777, 2
    qkv = _qkv(B, T, H, 99, dev, scale=0.5)
    gamma = cuda_ops.gammas(H, dev)
    g = torch.Generator(device=dev).manual_seed(5)
    s0 = 0.05 * torch.randn(B, H, 256, 256, generator=g, device=dev)
    _lib.set_option(0, "chunkwise_segments", nseg)
    try:
        out, ss, st = cuda_ops.retention_chunkwise_bf16(qkv, B, T, H, gamma, state_in=s0, chunk=chunk)
        torch.cuda.synchronize()
    finally:
        _lib.set_option(0, "chunkwise_segments", 0)
    assert _lib.check_device(0) == 0
    ref, S = _core_ref(qkv, B, T, H, s0.cpu().numpy().astype(np.float64))
    assert rel_err(out.float().cpu().numpy(), ref) < TOL
    assert rel_err(st.cpu().numpy(), S) < TOL
    assert rel_err(ss.cpu().numpy().sum(1), (ref * ref).sum(1)) < TOL


def test_gemm_bf16_kblocked_operand_and_blocked_parts(dev):
    """af_gemm_bf16 reading A as stacked K blocks [K/kb][M][kb] and row sums
    of squares as stacked blocks [P/pb][M][pb] equals the plain product."""
    from aceflow_b200 import cuda_ops

    M, N, K, kb, P, pb = 300, 192, 512, 128, 6, 3
    g = torch.Generator(device=dev).manual_seed(3)
    a = torch.randn(M, K, generator=g, device=dev).bfloat16()
    b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    parts = torch.rand(M, P, generator=g, device=dev) * 10
    a_blk = torch.cat([a[:, i * kb:(i + 1) * kb] for i in range(K // kb)], 0).contiguous()
    p_blk = torch.cat([parts[:, i * pb:(i + 1) * pb] for i in range(P // pb)], 0).contiguous()
    out = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a_blk, b, out, p_blk, inv_d=1.0 / K, eps=1e-6, a_kblock=kb, parts_block=pb)
    scale = 1.0 / torch.sqrt(parts.double().sum(1, keepdim=True) / K + 1e-6)
    ref = (a.double() @ b.double().t()) * scale
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    plain = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a, b, plain, parts, inv_d=1.0 / K, eps=1e-6)
    assert rel_err(plain.cpu().numpy(), ref.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("groups,layout,chunk", [(0, "columns", 64), (2, "columns", 64), (0, "rows", 64),
                                                 (0, "columns", 128), (0, "rows", 128)])
def test_head_sharded_prefill_single_rank(dev, groups, layout, chunk):
    """af_prefill_head_sharded (columns: all-gather; in one piece or as two
    head groups) and af_prefill_head_sharded_rows (rows: all-to-all) on a
    1-rank communicator equal the float64 layer and af_msr_prefill_bf16."""
    from aceflow_b200 import _lib, cuda_ops
    from aceflow_b200.sharded import HeadShardedPrefill

    B, T, H = 1, 600, 2
    d = H * 256
    rng = np.random.default_rng(21)
    tb = lambda a: torch.from_numpy(a).to(dev).bfloat16()  # noqa: E731
    x = tb(rng.standard_normal((B, T, d)).astype(np.float32))
    wqkv = tb((0.02 * rng.standard_normal((3 * d, d))).astype(np.float32))
    wo = tb((0.02 * rng.standard_normal((d, d))).astype(np.float32))
    rw = torch.from_numpy((1 + 0.1 * rng.standard_normal(d)).astype(np.float32)).to(dev)
    sp = HeadShardedPrefill(wqkv, wo, rw, H, 1e-6, layout=layout, chunk=chunk)
    _lib.set_option(0, "sharded_head_groups", groups)
    try:
        st = torch.empty(B, H, 256, 256, device=dev)
        out = sp(x, state_out=st)
        torch.cuda.synchronize()
        if layout == "rows":
            assert tuple(out.shape) == (B * T, d)
            out = sp.gather_output(out, B, T)
    finally:
        _lib.set_option(0, "sharded_head_groups", 0)
        sp.close()
    assert _lib.check_device(0) == 0
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    wq_, wk_, wv_ = np.split(f(wqkv), 3)
    ref = R.msr_forward64(f(x), wq_, wk_, wv_, f(wo), H, f(rw), 1e-6)
    assert rel_err(out.cpu().numpy(), ref) < TOL
    one, st1 = cuda_ops.msr_prefill_bf16(x, wqkv, wo, rw, cuda_ops.gammas(H, dev), 1e-6, chunk=chunk)
    assert rel_err(out.cpu().numpy(), one.cpu().numpy()) < 1e-3
    assert rel_err(st.cpu().numpy(), st1.cpu().numpy()) < 1e-3


# ---- the reference module API on CUDA: af.nn.MultiScaleRetention ----------
def _module(d, H, seed, **kw):
    import aceflow_b200 as af

    rng = np.random.default_rng(seed)
    m = af.nn.MultiScaleRetention(d, H, **kw)
    for name in ("w_q", "w_k", "w_v", "w_o"):
        w = torch.from_numpy((0.02 * rng.standard_normal((d, d))).astype(np.float32)).bfloat16().float().numpy()
        setattr(m, name, af.nn.Parameter(af.Tensor(w)))
    m.ret_norm.weight = af.nn.Parameter(af.Tensor((1 + 0.1 * rng.standard_normal(d)).astype(np.float32)))
    return m.to("cuda:0")


def _module_ref(m, x64):
    f = lambda p: p.numpy().astype(np.float64)  # noqa: E731
    return R.msr_forward64(x64, f(m.w_q), f(m.w_k), f(m.w_v), f(m.w_o), m.num_heads, f(m.ret_norm.weight), 1e-6)


def test_module_bf16_input_runs_tensor_core_prefill(dev):
    """A bf16 prompt through af.nn.MultiScaleRetention(...).to('cuda') takes
    the tensor-core chunkwise prefill: bf16 output within 2e-2 of float64,
    and library launches (no host arithmetic)."""
    import aceflow_b200 as af
    from aceflow_b200 import _lib

    B, T, d, H = 2, 150, 512, 2
    m = _module(d, H, 61)
    x = torch.from_numpy(np.random.default_rng(62).standard_normal((B, T, d)).astype(np.float32)).to(dev).bfloat16()
    n0 = _lib.launch_count(0)
    out = m(af.Tensor(x, device="cuda:0", dtype="bfloat16"))
    assert _lib.launch_count(0) - n0 >= 3  # QKV GEMM, chunkwise kernel, W_o GEMM
    assert out.dtype == "bfloat16"
    assert rel_err(out.numpy(), _module_ref(m, x.float().cpu().numpy())) < TOL


def test_module_fp32_input_exact_by_default_and_tensor_cores_on_request(dev):
    """fp32 prompts: the exact fp32 path by default (1e-4 of float64); with
    prefill_dtype='bfloat16' the tensor-core path (2e-2), output fp32."""
    import aceflow_b200 as af

    B, T, d, H = 2, 130, 512, 2
    x = np.random.default_rng(63).standard_normal((B, T, d)).astype(np.float32)
    exact = _module(d, H, 64)
    ref = _module_ref(exact, x)
    out = exact(af.Tensor(x, device="cuda:0"))
    assert out.dtype == "float32" and rel_err(out.numpy(), ref) < 1e-4
    tc = _module(d, H, 64, prefill_dtype="bfloat16")
    out = tc(af.Tensor(x, device="cuda:0"))
    assert out.dtype == "float32" and rel_err(out.numpy(), ref) < TOL


def test_module_forward_chunkwise_state_hands_over_to_decode(dev):
    """forward_chunkwise over two prompt pieces (the second from the first's
    state), then forward_recurrent steps from the returned state, equal the
    float64 forward over the whole sequence."""
    import aceflow_b200 as af

    B, d, H, T1, T2, n = 2, 512, 2, 100, 77, 3
    m = _module(d, H, 65)
    x = np.random.default_rng(66).standard_normal((B, T1 + T2 + n, d)).astype(np.float32)
    xb = torch.from_numpy(x).bfloat16().float().numpy()  # the values the bf16 prefill reads
    ref = _module_ref(m, xb)
    t = lambda a: af.Tensor(np.ascontiguousarray(a), device="cuda:0", dtype="bfloat16")  # noqa: E731
    o1, st = m.forward_chunkwise(t(xb[:, :T1]))
    o2, st = m.forward_chunkwise(t(xb[:, T1:T1 + T2]), state=st)
    assert st.shape == [B, H, 256, 256]
    assert rel_err(np.concatenate([o1.numpy(), o2.numpy()], 1), ref[:, :T1 + T2]) < TOL
    outs = []
    for i in range(n):
        o, st = m.forward_recurrent(af.Tensor(xb[:, T1 + T2 + i], device="cuda:0"), st)
        outs.append(o.numpy())
    assert rel_err(np.stack(outs, 1), ref[:, T1 + T2:]) < TOL


def test_module_forward_chunkwise_needs_head_dim_256(dev):
    import aceflow_b200 as af

    m = af.nn.MultiScaleRetention(64, 4).to("cuda:0")
    with pytest.raises(ValueError, match="head_dim 256"):
        m.forward_chunkwise(af.Tensor(np.zeros((1, 8, 64), np.float32), device="cuda:0"))
    with pytest.raises(ValueError, match="chunk"):
        _module(512, 2, 1).forward_chunkwise(af.Tensor(np.zeros((1, 8, 512), np.float32), device="cuda:0"), chunk=48)


# ---- backward of the chunkwise form ---------------------------------------
@pytest.mark.parametrize("B,T,H,with_state", [(1, 128, 1, False), (2, 200, 2, True), (1, 777, 2, True),
                                              (3, 65, 1, False), (1, 300, 1, False), (2, 300, 1, True),
                                              (1, 1, 1, True), (2, 3, 2, False)])
def test_chunkwise_backward_matches_float64_gradients(dev, B, T, H, with_state):
    """dQ, dK, dV and the initial state's gradient of the chunkwise kernel
    (three passes of the 128-token kernel, two over reversed time) against
    the float64 closed form of the parallel form's gradients; 2e-2 each."""
    from aceflow_b200 import _lib, cuda_ops

    d = H * 256
    qkv = _qkv(B, T, H, 300 + T, dev, scale=0.5)
    g = torch.Generator(device=dev).manual_seed(301)
    dout = torch.randn(B * T, d, generator=g, device=dev).bfloat16()
    s0 = 0.05 * torch.randn(B, H, 256, 256, generator=g, device=dev) if with_state else None
    gamma = cuda_ops.gammas(H, dev)
    dqkv, dS = cuda_ops.retention_chunkwise_backward_bf16(qkv, dout, B, T, H, gamma, state_in=s0, want_dstate=True)
    torch.cuda.synchronize()
    assert _lib.check_device(0) == 0
    a = qkv.float().cpu().numpy().astype(np.float64).reshape(B, T, 3, H, 256)
    q, k, v = (a[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    do = dout.float().cpu().numpy().astype(np.float64).reshape(B, T, H, 256).transpose(0, 2, 1, 3)
    ref = R.retention_backward64(q, k, v, R.gammas(H), do, None if s0 is None else s0.cpu().numpy())
    got = dqkv.float().cpu().numpy().reshape(B, T, 3, H, 256)
    for i, name in enumerate(("dq", "dk", "dv")):
        assert rel_err(got[:, :, i].transpose(0, 2, 1, 3), ref[i]) < TOL, name
    assert rel_err(dS.cpu().numpy(), ref[3]) < TOL


def test_chunkwise_backward_matches_finite_differences_of_the_forward(dev):
    """Along the direction of the GPU's own gradient g, the oracle forward's
    loss <dO, O(x + e g)> changes by e <g_true, g>, which must equal |g|^2
    to within 2e-2 (central differences in float64; along g the sum has no
    cancellation, so bf16 rounding of single entries cannot dominate it)."""
    from aceflow_b200 import cuda_ops

    B, T, H = 1, 300, 1
    qkv = _qkv(B, T, H, 311, dev, scale=0.5)
    g0 = torch.Generator(device=dev).manual_seed(312)
    dout = torch.randn(B * T, 256, generator=g0, device=dev).bfloat16()
    dqkv, _ = cuda_ops.retention_chunkwise_backward_bf16(qkv, dout, B, T, H, cuda_ops.gammas(H, dev))
    a = qkv.float().cpu().numpy().astype(np.float64).reshape(B, T, 3, H, 256).transpose(2, 0, 3, 1, 4)
    do = dout.float().cpu().numpy().astype(np.float64).reshape(B, T, H, 256).transpose(0, 2, 1, 3)
    g = dqkv.float().cpu().numpy().astype(np.float64).reshape(B, T, 3, H, 256).transpose(2, 0, 3, 1, 4)
    dirs = g / np.linalg.norm(g)
    eps = 1e-3
    f = lambda x: float((R.retention_chunkwise64(x[0], x[1], x[2], R.gammas(H), 64)[0] * do).sum())  # noqa: E731
    fd = (f(a + eps * dirs) - f(a - eps * dirs)) / (2 * eps)
    an = float((g * dirs).sum())
    assert abs(an - fd) <= 2e-2 * abs(fd)


def test_chunkwise_autograd_function(dev):
    """retention_chunkwise_autograd: loss.backward() through the tensor-core
    forward gives the float64 closed-form gradient of the parallel form."""
    from aceflow_b200 import cuda_ops

    B, T, H = 2, 150, 1
    qkv = _qkv(B, T, H, 321, dev, scale=0.5).requires_grad_(True)
    g = torch.Generator(device=dev).manual_seed(322)
    w = torch.randn(B * T, H * 256, generator=g, device=dev)
    out = cuda_ops.retention_chunkwise_autograd(qkv, B, T, H, cuda_ops.gammas(H, dev))
    (out.float() * w).sum().backward()
    a = qkv.detach().float().cpu().numpy().astype(np.float64).reshape(B, T, 3, H, 256)
    q, k, v = (a[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    do = w.bfloat16().double().cpu().numpy().reshape(B, T, H, 256).transpose(0, 2, 1, 3)
    ref = R.retention_backward64(q, k, v, R.gammas(H), do)
    got = qkv.grad.float().cpu().numpy().reshape(B, T, 3, H, 256)
    for i in range(3):
        assert rel_err(got[:, :, i].transpose(0, 2, 1, 3), ref[i]) < TOL
