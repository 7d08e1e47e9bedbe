"""af.ops functional API (mirrors aceflow/ops/functional.py:14-53).

CUDA tensors run in libaceflow_cuda.so; CPU tensors keep the reference's
numpy formulas.  gelu/softmax are off the retention path and CPU-only.
"""
from __future__ import annotations

import numpy as np

from ..core.tensor import Tensor


def _ops():
    from .. import cuda_ops

    return cuda_ops


def matmul(a: Tensor, b: Tensor) -> Tensor:
    return a.matmul(b)


def rms_norm(x: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    if x.device.is_cuda:
        return Tensor._wrap(_ops().rms_norm(x.torch, weight.torch, eps), x.device)
    arr = x.numpy()
    variance = np.mean(np.square(arr), axis=-1, keepdims=True)
    return Tensor(arr / np.sqrt(variance + eps) * weight.numpy(), x.device)


def swiglu(x: Tensor, w_gate: Tensor, w_up: Tensor, w_down: Tensor) -> Tensor:
    if x.device.is_cuda:
        ops = _ops()
        gate = ops.linear(x.torch, w_gate.torch)
        up = ops.linear(x.torch, w_up.torch)
        return Tensor._wrap(ops.linear(ops.silu_mul(gate, up), w_down.torch), x.device)
    arr = x.numpy()
    gate = np.matmul(arr, w_gate.numpy().T)
    up = np.matmul(arr, w_up.numpy().T)
    return Tensor(np.matmul(gate / (1.0 + np.exp(-gate)) * up, w_down.numpy().T), x.device)


def silu(x: Tensor) -> Tensor:
    if x.device.is_cuda:
        return Tensor._wrap(_ops().silu_mul(x.torch), x.device)
    arr = x.numpy()
    return Tensor(arr / (1.0 + np.exp(-arr)), x.device)


def gelu(x: Tensor) -> Tensor:
    if x.device.is_cuda:
        raise NotImplementedError("gelu is not part of the retention hot path (no CUDA kernel)")
    arr = x.numpy()
    cdf = 0.5 * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (arr + 0.044715 * np.power(arr, 3))))
    return Tensor(arr * cdf, x.device)


def softmax(x: Tensor, axis: int = -1) -> Tensor:
    if x.device.is_cuda:
        raise NotImplementedError("softmax is not part of the retention hot path (no CUDA kernel)")
    arr = x.numpy()
    e_x = np.exp(arr - np.max(arr, axis=axis, keepdims=True))
    return Tensor(e_x / np.sum(e_x, axis=axis, keepdims=True), x.device)
