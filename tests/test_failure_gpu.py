"""Failure detection on the GPU without a fault: a bounded device-side wait
is made to run out (an mbarrier phase nothing completes, a 50 ms limit); the
kernel returns, the host reads AF_ERR_TIMEOUT through af_check_device, and
the same context keeps computing correct results afterwards."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
LIMIT_NS = 50_000_000  # 50 ms


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def test_bounded_wait_times_out_with_a_status(dev):
    from aceflow_b200 import _lib, cuda_ops
    from oracle import cpu_ref
    from oracle import retention_ref as R

    ctx = _lib.context(0)
    assert _lib.check_device(0) == 0
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.call("af_selftest_bounded_wait", ctx, LIMIT_NS, stream)
    flags = ctypes.c_int()
    rc = _lib.lib().af_check_device(ctx, ctypes.byref(flags), 0)
    assert rc == _lib.AF_ERR_TIMEOUT and flags.value & (1 << _lib.AF_ERR_TIMEOUT)
    assert "timed out" in _lib.last_error()
    with pytest.raises(RuntimeError, match="timed out"):
        _lib.check_device(0, reset=True)  # reads it once more, then clears it
    assert _lib.check_device(0) == 0
    # the context (and the GPU) still compute: one decode step against the oracle
    rng = np.random.default_rng(71)
    B, d, H = 4, 512, 2
    w_qkv = (0.02 * rng.standard_normal((3 * d, d))).astype(np.float32)
    w_o = (0.02 * rng.standard_normal((d, d))).astype(np.float32)
    rw = np.ones(d, np.float32)
    gamma = R.gammas(H)
    st = np.zeros((B, H, d // H, d // H), np.float32)
    x = rng.standard_normal((B, d)).astype(np.float32)
    ref = cpu_ref.msr_decode_step(x, st, gamma, w_qkv, w_o, rw, 1e-6)
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    out = cuda_ops.msr_decode_step(t(x), torch.zeros(B, H, d // H, d // H, device=dev), t(gamma), t(w_qkv), t(w_o),
                                   t(rw), 1e-6)
    assert rel_err(out.cpu().numpy(), ref) < 1e-4
    assert _lib.check_device(0) == 0


def test_selftest_rejects_limits_outside_its_range(dev):
    from aceflow_b200 import _lib

    for bad in (0, 999, 3_000_000_000):
        with pytest.raises(ValueError, match="limit_ns"):
            _lib.call("af_selftest_bounded_wait", _lib.context(0), bad, None)
