"""Tensor-core (tcgen05) GEMM parity, through the C ABI.

bf16 operands: compared with an fp64 product of the same bf16 values (the
only difference is fp32 accumulation order).  fp32 operands (3xTF32 split):
compared with fp64, must hold fp32-level accuracy (<= 1e-5 relative).
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _check(dev):
    from aceflow_b200 import _lib

    assert _lib.check_device(0) == 0


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (1, 16, 8), (300, 200, 136), (256, 6144, 2048),
                                   (4096, 2048, 2048), (77, 512, 1000)])
def test_bf16_gemm_matches_fp64(dev, M, N, K):
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g, device=dev).bfloat16()
    w = (0.02 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    b = torch.randn(N, generator=g, device=dev)
    y = cuda_ops.linear_bf16(x, w, b)
    ref = x.double() @ w.double().T + b.double()
    assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    yb = cuda_ops.linear_bf16(x, w, out_dtype=torch.bfloat16)
    assert rel_err(yb.float().cpu().numpy(), (x.double() @ w.double().T).cpu().numpy()) < 1e-2
    _check(dev)


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (256, 6144, 2048), (256, 2048, 2048), (3, 40, 48),
                                   (130, 2048, 5632), (1000, 264, 96)])
def test_tf32x3_gemm_is_fp32_accurate(dev, M, N, K):
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N * 3 + K)
    x = torch.randn(M, K, generator=g, device=dev)
    w = 0.02 * torch.randn(N, K, generator=g, device=dev)
    y = cuda_ops.linear(x, w)
    ref = x.double() @ w.double().T
    err = rel_err(y.cpu().numpy(), ref.cpu().numpy())
    assert err < 1e-5, err
    _check(dev)


def test_unaligned_k_uses_simt_path(dev):
    from aceflow_b200 import cuda_ops

    x = torch.randn(5, 13, device=dev)
    w = torch.randn(7, 13, device=dev)
    assert rel_err(cuda_ops.linear(x, w).cpu().numpy(), (x.double() @ w.double().T).cpu().numpy()) < 1e-6


@pytest.mark.parametrize("bn", ["96", "128", "64", "32"])
@pytest.mark.parametrize("M,N,K", [(256, 6144, 2048), (200, 1000, 512), (1, 96, 64)])
def test_presplit_gemm_every_tile_width(dev, bn, M, N, K, monkeypatch):
    """The pre-split 3xTF32 GEMM (decode projections) at each tile width,
    the 96-wide tile included, is fp32-accurate."""
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g, device=dev)
    w = 0.02 * torch.randn(N, K, generator=g, device=dev)
    ref = (x.double() @ w.double().T).cpu().numpy()
    monkeypatch.setenv("AF_GEMM_BN", bn)
    y = cuda_ops.linear_f32_split(cuda_ops.split_tf32(x), cuda_ops.split_tf32(w))
    torch.cuda.synchronize()
    monkeypatch.delenv("AF_GEMM_BN")
    assert rel_err(y.cpu().numpy(), ref) < 1e-5
    _check(dev)


@pytest.mark.parametrize("M,N,K,pad", [(300, 192, 256, 0), (129, 200, 128, 1), (4096, 512, 1024, 0)])
def test_bf16_gemm_bias_residual_epilogue(dev, M, N, K, pad):
    """Bias and residual in the epilogue, with the residual in vector
    (aligned row stride) and scalar (odd row stride) form, and in place."""
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device=dev).bfloat16()
    b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    bias = torch.randn(N, generator=g, device=dev)
    base = torch.randn(M, N + pad, generator=g, device=dev)
    res = base[:, :N]
    ref = a.double() @ b.double().t() + bias.double() + res.double()
    out = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a, b, out, bias=bias, residual=res)
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    # in place: out is the residual
    inplace = res.clone()
    cuda_ops.gemm_bf16(a, b, inplace, bias=bias, residual=inplace)
    assert rel_err(inplace.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    _check(dev)


@pytest.mark.parametrize("M,N,K", [(8192, 2048, 2048), (8292, 2112, 1000)])
def test_bf16_gemm_cta_pair_matches_fp64(dev, M, N, K):
    """Large bf16 GEMMs run on CTA pairs (cta_group::2, 256 x 256 tiles):
    ragged M, N, K, with bias, residual and the 1/rms row scale, equal to the
    fp64 product and to the one-SM persistent kernel."""
    from aceflow_b200 import _lib, cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device=dev).bfloat16()
    b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    bias = torch.randn(N, generator=g, device=dev)
    res = torch.randn(M, N, generator=g, device=dev)
    parts = torch.rand(M, 3, generator=g, device=dev) * 10
    scale = 1.0 / torch.sqrt(parts.double().sum(1, keepdim=True) / K + 1e-6)
    ref = (a.double() @ b.double().t()) * scale + bias.double() + res.double()
    out = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a, b, out, parts, inv_d=1.0 / K, eps=1e-6, bias=bias, residual=res)
    torch.cuda.synchronize()
    _check(dev)
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    _lib.set_option(0, "gemm_pair", 0)
    try:
        one = torch.empty(M, N, device=dev)
        cuda_ops.gemm_bf16(a, b, one, parts, inv_d=1.0 / K, eps=1e-6, bias=bias, residual=res)
        torch.cuda.synchronize()
    finally:
        _lib.set_option(0, "gemm_pair", 1)
    assert rel_err(out.cpu().numpy(), one.cpu().numpy()) < 1e-6
    _check(dev)


@pytest.mark.parametrize("producers", [2, 4])
def test_gemm_producer_threads_same_result(dev, producers):
    """TMA loads spread over several producer threads (af_set_option
    "gemm_producers") feed the MMAs the same K slices in the same order: the
    CTA-pair GEMM (no split-K) is bit-identical, the split-K ones (atomic
    adds in any order) and the pre-split decode GEMM agree to fp32 rounding.
    Kernels whose ring is shallower than the producer count (3 stages for
    3xTF32 tiles of 128 columns) cap it."""
    from aceflow_b200 import _lib, cuda_ops

    g = torch.Generator(device=dev).manual_seed(producers)
    cases = []
    for M, N, K in [(8192, 2048, 2048), (300, 200, 136), (64, 11264, 2048)]:
        a = torch.randn(M, K, generator=g, device=dev).bfloat16()
        b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
        cases.append((a, b))
    x = torch.randn(256, 2048, generator=g, device=dev)
    w = 0.02 * torch.randn(6144, 2048, generator=g, device=dev)
    xs, ws = cuda_ops.split_tf32(x), cuda_ops.split_tf32(w)

    def run():
        outs = []
        for a, b in cases:
            o = torch.empty(a.shape[0], b.shape[0], device=dev)
            cuda_ops.gemm_bf16(a, b, o)
            outs.append(o)
        outs.append(cuda_ops.linear_f32_split(xs, ws))
        torch.cuda.synchronize()
        return outs

    ref = run()
    _lib.set_option(0, "gemm_producers", producers)
    try:
        got = run()
    finally:
        _lib.set_option(0, "gemm_producers", 1)
    assert torch.equal(ref[0], got[0])
    for r, o in zip(ref[1:], got[1:]):
        assert rel_err(o.cpu().numpy(), r.cpu().numpy()) < 1e-6
    _check(dev)


@pytest.mark.parametrize("bn", ["16", "32", "64", "128"])
@pytest.mark.parametrize("M,N,K", [(64, 11264, 2048), (300, 200, 192), (1000, 96, 4096)])
def test_bf16_two_k_slices_per_stage(dev, bn, M, N, K, monkeypatch):
    """bf16 tiles up to 128 wide load two 64-element K slices per ring stage
    with one 3-D TMA copy per operand (K a multiple of 64): the MMAs run in
    the same order as with one slice per stage, so without split-K the two
    are bit-identical, and both equal the fp64 product."""
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device=dev).bfloat16()
    b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    ref = (a.double() @ b.double().t()).cpu().numpy()
    monkeypatch.setenv("AF_GEMM_BN", bn)
    monkeypatch.setenv("AF_GEMM_SPLITS", "1")
    outs = []
    for ks in ("2", "1"):
        monkeypatch.setenv("AF_GEMM_KS", ks)
        o = torch.empty(M, N, device=dev)
        cuda_ops.gemm_bf16(a, b, o)
        torch.cuda.synchronize()
        outs.append(o)
    assert torch.equal(outs[0], outs[1])
    assert rel_err(outs[0].cpu().numpy(), ref) < 1e-5
    # split-K over two-slice stages (atomics): fp32 rounding of the partial sums
    monkeypatch.setenv("AF_GEMM_KS", "2")
    monkeypatch.setenv("AF_GEMM_SPLITS", "3")
    o = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a, b, o)
    torch.cuda.synchronize()
    assert rel_err(o.cpu().numpy(), ref) < 1e-5
    _check(dev)


@pytest.mark.parametrize("M,N,K,bn,splits", [(256, 2048, 2048, "128", "4"), (300, 200, 512, "64", "3"),
                                             (130, 1000, 1024, "32", "2")])
def test_staged_reduce_add_epilogue(dev, M, N, K, bn, splits, monkeypatch):
    """Split-K partial products added into the output by TMA reduce-adds of
    128-byte-swizzled shared-memory boxes (ragged M and N clipped by the
    tensor map), with and without the 1/rms row scale, equal to the per-thread
    atomics and to fp64."""
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N)
    x = torch.randn(M, K, generator=g, device=dev)
    w = 0.02 * torch.randn(N, K, generator=g, device=dev)
    parts = torch.rand(M, 4, generator=g, device=dev) * 10
    scale = 1.0 / torch.sqrt(parts.double().sum(1, keepdim=True) / K + 1e-6)
    xs, ws = cuda_ops.split_tf32(x), cuda_ops.split_tf32(w)
    ref = (x.double() @ w.double().T).cpu().numpy()
    monkeypatch.setenv("AF_GEMM_BN", bn)
    monkeypatch.setenv("AF_GEMM_SPLITS", splits)
    outs = []
    for no_stage in (False, True):
        if no_stage:
            monkeypatch.setenv("AF_GEMM_NO_STAGE", "1")
        y = cuda_ops.linear_f32_split(xs, ws)
        torch.cuda.synchronize()
        outs.append(y.cpu().numpy())
    assert rel_err(outs[0], ref) < 1e-5
    assert rel_err(outs[0], outs[1]) < 1e-6
    monkeypatch.delenv("AF_GEMM_NO_STAGE")
    ab = x.bfloat16()
    bb = w.bfloat16()
    o = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(ab, bb, o, parts, inv_d=1.0 / K, eps=1e-6)
    torch.cuda.synchronize()
    ref2 = (ab.double() @ bb.double().t() * scale).cpu().numpy()
    assert rel_err(o.cpu().numpy(), ref2) < 1e-5
    _check(dev)


@pytest.mark.parametrize("M,N,K", [(8292, 2112, 2048), (4096, 768, 4096)])
def test_pair_gemm_staged_store_epilogue(dev, M, N, K, monkeypatch):
    """CTA-pair GEMM with fp32 and bf16 output written through
    128-byte-swizzled shared-memory boxes and TMA stores (two K slices per
    stage leave room for 8 KB per epilogue warp): ragged M and N, bias and
    1/rms row scale, and an in-place residual added by TMA reduce-adds:
    every element written, equal to the per-thread stores up to rounding and
    to fp64."""
    from aceflow_b200 import cuda_ops

    g = torch.Generator(device=dev).manual_seed(M + N)
    a = torch.randn(M, K, generator=g, device=dev).bfloat16()
    b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    bias = torch.randn(N, generator=g, device=dev)
    parts = torch.rand(M, 2, generator=g, device=dev) * 10
    scale = 1.0 / torch.sqrt(parts.double().sum(1, keepdim=True) / K + 1e-6)
    ref = ((a.double() @ b.double().t()) * scale + bias.double()).cpu().numpy()
    outs = []
    for no_stage in (False, True):
        if no_stage:
            monkeypatch.setenv("AF_GEMM_NO_STAGE", "1")
        o = torch.full((M, N), float("nan"), device=dev)
        cuda_ops.gemm_bf16(a, b, o, parts, inv_d=1.0 / K, eps=1e-6, bias=bias)
        torch.cuda.synchronize()
        outs.append(o)
    assert torch.isfinite(outs[0]).all()  # every element written (the buffer started as NaN)
    assert rel_err(outs[0].cpu().numpy(), outs[1].cpu().numpy()) < 1e-6  # same products, FMA contraction aside
    assert rel_err(outs[0].cpu().numpy(), ref) < 1e-5
    # in place (x += ...): the output holds the residual; the staged tile is
    # added into it by TMA reduce-adds
    res = torch.randn(M, N, generator=g, device=dev)
    inplace = []
    for no_stage in (True, False):
        if not no_stage:
            monkeypatch.delenv("AF_GEMM_NO_STAGE")
        o = res.clone()
        cuda_ops.gemm_bf16(a, b, o, parts, inv_d=1.0 / K, eps=1e-6, bias=bias, residual=o)
        torch.cuda.synchronize()
        inplace.append(o)
    ref_ip = ref + res.double().cpu().numpy()
    assert rel_err(inplace[1].cpu().numpy(), ref_ip) < 1e-5
    assert rel_err(inplace[1].cpu().numpy(), inplace[0].cpu().numpy()) < 1e-6
    # bf16 output: one [32 x 64] box per 64 columns, double-buffered
    yb = cuda_ops.linear_bf16(a, b, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    monkeypatch.setenv("AF_GEMM_NO_STAGE", "1")
    yb2 = cuda_ops.linear_bf16(a, b, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.isfinite(yb.float()).all()
    assert rel_err(yb.float().cpu().numpy(), yb2.float().cpu().numpy()) < 1e-2
    assert rel_err(yb.float().cpu().numpy(), (a.double() @ b.double().t()).cpu().numpy()) < 1e-2
    _check(dev)


@pytest.mark.parametrize("kb", [256, 64])
def test_pair_gemm_kblocked_operand(dev, kb):
    """CTA-pair GEMM reading A as stacked K blocks [K/kb][M][kb] (the
    head-sharded prefill's all-gathered outputs): K blocks that are multiples
    of 128 take two-slice stages with 3-D copies, others one slice; both
    equal the plain product."""
    from aceflow_b200 import cuda_ops

    M, N, K = 8192, 2560, 1024
    g = torch.Generator(device=dev).manual_seed(kb)
    a = torch.randn(M, K, generator=g, device=dev).bfloat16()
    b = (0.05 * torch.randn(N, K, generator=g, device=dev)).bfloat16()
    a_blk = torch.cat([a[:, i * kb:(i + 1) * kb] for i in range(K // kb)], 0).contiguous()
    out = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a_blk, b, out, a_kblock=kb)
    ref = torch.empty(M, N, device=dev)
    cuda_ops.gemm_bf16(a, b, ref)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < 1e-6
    assert rel_err(out.cpu().numpy(), (a.double() @ b.double().t()).cpu().numpy()) < 1e-5
    _check(dev)
