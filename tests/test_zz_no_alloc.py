"""The allocation-free decode step (af_msr_decode_step_f32_noalloc).

Callers that cannot allocate device memory when they run a step (inside a
CUDA-graph capture, or under their own arena allocator) use this entry point;
it keeps its scratch in a fixed array inside the library.  This file runs
last (pytest collects it last) and must pass alone in a fresh process as
well as after the other tests: the first call on the device does the
one-time set-up either way.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4  # the fp32 tolerance of the decode tests


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def test_noalloc_step_matches_allocating_step_twice(dev):
    """Two consecutive steps through the C ABI: the static-scratch entry
    point gives the same output and state as af_msr_decode_step_f32."""
    from aceflow_b200 import _lib, cuda_ops

    B, d, H = 64, 2048, 8
    g = torch.Generator(device=dev).manual_seed(123)
    w_qkv = 0.02 * torch.randn(3 * d, d, generator=g, device=dev)
    w_o = 0.02 * torch.randn(d, d, generator=g, device=dev)
    rw = 1 + 0.1 * torch.randn(d, generator=g, device=dev)
    gamma = cuda_ops.gammas(H, dev)
    st_ref = torch.zeros(B, H, d // H, d // H, device=dev)
    st_new = torch.zeros_like(st_ref)
    for _ in range(2):
        x = torch.randn(B, d, generator=g, device=dev)
        ref = cuda_ops.msr_decode_step(x, st_ref, gamma, w_qkv, w_o, rw, 1e-6)
        got = cuda_ops.msr_decode_step_noalloc(x, st_new, gamma, w_qkv, w_o, rw, 1e-6)
        torch.cuda.synchronize()
        assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) < TOL
        assert rel_err(st_new.cpu().numpy(), st_ref.cpu().numpy()) < TOL
    assert _lib.check_device(0) == 0


def test_noalloc_rejects_batches_beyond_the_static_scratch(dev):
    from aceflow_b200 import _lib

    d, H = 2048, 8
    too_many = (1 << 22) // (4 * d + H) + 1
    with pytest.raises(ValueError, match="static array"):
        _lib.call("af_msr_decode_step_f32_noalloc", 16, 16, 16, 16, 16, 16, 1e-6, too_many, d, H, 16, None)
