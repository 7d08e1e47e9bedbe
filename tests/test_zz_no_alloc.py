"""The allocation-free decode step (af_msr_decode_step_f32_noalloc).

Who needs it: a serving process that carves its device memory up front with
its own arena allocator, or a plugin inside a host that owns the GPU's memory
budget, cannot let the library call cudaMalloc when a step runs.  This entry
point keeps its scratch in a fixed array inside the library instead (16 MiB,
batch * (4 * d_model + heads) floats at most).

Checked here through the C ABI: two steps in a row against the C oracle (the
reference's CPU decode step) and against the allocating entry point, at 64
streams and at the largest batch the array holds for d_model 2048 (511);
512 streams are rejected; the entry point's own device error word reads back
as 0, and a bounded wait made to run out sets it; and the device's free
memory does not change across a call.  This file
runs last (pytest collects it last) and passes alone in a fresh process as
well as after the other tests: the first call on the device does the one-time
set-up either way.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4  # the fp32 tolerance of the decode tests
D, H = 2048, 8
CAPACITY = 1 << 22  # floats in the library's static scratch array


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _weights(seed):
    rng = np.random.default_rng(seed)
    w_qkv = (0.02 * rng.standard_normal((3 * D, D))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((D, D))).astype(np.float32)
    rw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return rng, w_qkv, w_o, rw


@pytest.mark.parametrize("B", [64, 511])
def test_noalloc_step_matches_oracle_and_allocating_step_twice(dev, B):
    """Two consecutive steps: the static-scratch entry point equals the C
    oracle (max rel err <= 1e-4) and af_msr_decode_step_f32, output and
    state; its error word stays clear."""
    from aceflow_b200 import cuda_ops
    from oracle import cpu_ref
    from oracle import retention_ref as R

    assert B * (4 * D + H) <= CAPACITY
    rng, w_qkv, w_o, rw = _weights(B)
    gamma = R.gammas(H)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    wq_d, wo_d, rw_d, g_d = t(w_qkv), t(w_o), t(rw), t(gamma)
    st_host = np.zeros((B, H, D // H, D // H), np.float32)
    st_alloc = torch.zeros(B, H, D // H, D // H, device=dev)
    st_new = torch.zeros_like(st_alloc)
    out = torch.empty(B, D, device=dev)
    for _ in range(2):
        x = rng.standard_normal((B, D)).astype(np.float32)
        ref = cpu_ref.msr_decode_step(x, st_host, gamma, w_qkv, w_o, rw, 1e-6)
        x_d = t(x)
        alloc = cuda_ops.msr_decode_step(x_d, st_alloc, g_d, wq_d, wo_d, rw_d, 1e-6)
        got = cuda_ops.msr_decode_step_noalloc(x_d, st_new, g_d, wq_d, wo_d, rw_d, 1e-6, out=out)
        torch.cuda.synchronize()
        assert rel_err(got.cpu().numpy(), ref) < TOL
        assert rel_err(got.cpu().numpy(), alloc.cpu().numpy()) < TOL
        assert rel_err(st_new.cpu().numpy(), st_host) < TOL
    assert cuda_ops.noalloc_check_device(dev) == 0


def test_noalloc_call_leaves_free_memory_unchanged(dev):
    """After a first call (which loads the kernels), a further call changes
    the device's free memory by nothing."""
    from aceflow_b200 import cuda_ops

    B = 32
    _, w_qkv, w_o, rw = _weights(3)
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    wq_d, wo_d, rw_d, g_d = t(w_qkv), t(w_o), t(rw), cuda_ops.gammas(H, dev)
    st = torch.zeros(B, H, D // H, D // H, device=dev)
    x = torch.randn(B, D, device=dev)
    out = torch.empty(B, D, device=dev)
    cuda_ops.msr_decode_step_noalloc(x, st, g_d, wq_d, wo_d, rw_d, 1e-6, out=out)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    cuda_ops.msr_decode_step_noalloc(x, st, g_d, wq_d, wo_d, rw_d, 1e-6, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0
    assert cuda_ops.noalloc_check_device(dev) == 0


def test_noalloc_error_word_reports_a_timed_out_wait(dev):
    """The entry point's kernels report a bounded-wait timeout in its own
    device error word: a wait made to run out (50 ms limit, nothing arrives)
    sets it, af_check_device(NULL, ...) reports and clears it, and the next
    step is correct."""
    from aceflow_b200 import _lib, cuda_ops

    with torch.cuda.device(dev):
        _lib.call("af_selftest_bounded_wait", None, 50_000_000, torch.cuda.current_stream(dev).cuda_stream)
    with pytest.raises(RuntimeError, match="timed out"):
        cuda_ops.noalloc_check_device(dev)  # reads the word and clears it
    assert cuda_ops.noalloc_check_device(dev) == 0
    B = 16
    _, w_qkv, w_o, rw = _weights(5)
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    x = torch.randn(B, D, device=dev)
    st_a, st_b = torch.zeros(B, H, D // H, D // H, device=dev), torch.zeros(B, H, D // H, D // H, device=dev)
    g = cuda_ops.gammas(H, dev)
    ref = cuda_ops.msr_decode_step(x, st_a, g, t(w_qkv), t(w_o), t(rw), 1e-6)
    got = cuda_ops.msr_decode_step_noalloc(x, st_b, g, t(w_qkv), t(w_o), t(rw), 1e-6)
    torch.cuda.synchronize()
    assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) < TOL
    assert cuda_ops.noalloc_check_device(dev) == 0


def test_noalloc_rejects_batches_beyond_the_static_scratch(dev):
    """512 streams at d_model 2048 need more than the array holds: AF_ERR_ARG
    (ValueError) before any launch."""
    from aceflow_b200 import _lib

    too_many = CAPACITY // (4 * D + H) + 1
    assert too_many == 512
    with pytest.raises(ValueError, match="static array"):
        _lib.call("af_msr_decode_step_f32_noalloc", 16, 16, 16, 16, 16, 16, 1e-6, too_many, D, H, 16, None)
