"""Linear / RMSNorm / LayerNorm / SwiGLU (mirrors aceflow/nn/layers.py:11-88).

Initialisation draws from ``np.random`` in the reference's order, so a
seeded script builds identical weights with either package.  On a CUDA
device every forward runs in libaceflow_cuda.so; on the CPU the reference's
numpy formulas apply unchanged.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np

from ..core.tensor import Tensor
from .module import Module, Parameter


def _cuda_ops():
    from .. import cuda_ops

    return cuda_ops


class Linear(Module):
    """Fully connected layer: y = x A^T + b (layers.py:11-33)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        k = 1.0 / math.sqrt(in_features)
        self.weight = Parameter(Tensor(np.random.uniform(-k, k, (out_features, in_features)).astype(np.float32)))
        if bias:
            self.bias = Parameter(Tensor(np.random.uniform(-k, k, (out_features,)).astype(np.float32)))
        else:
            self.bias = None

    def forward(self, x: Tensor) -> Tensor:
        if x.device.is_cuda:
            b = None if self.bias is None else self.bias.torch
            return Tensor._wrap(_cuda_ops().linear(x.torch, self.weight.torch, b), x.device)
        out = np.matmul(x.numpy(), self.weight.numpy().T)
        if self.bias is not None:
            out = out + self.bias.numpy()
        return Tensor(out, x.device)


class RMSNorm(Module):
    """Root Mean Square Layer Normalization (layers.py:36-49), eps 1e-6."""

    def __init__(self, d_model: int, eps: float = 1e-6):
        super().__init__()
        self.d_model = d_model
        self.eps = eps
        self.weight = Parameter(Tensor(np.ones(d_model, dtype=np.float32)))

    def forward(self, x: Tensor) -> Tensor:
        if x.device.is_cuda:
            return Tensor._wrap(_cuda_ops().rms_norm(x.torch, self.weight.torch, self.eps), x.device)
        arr = x.numpy()
        rms = np.sqrt(np.mean(np.square(arr), axis=-1, keepdims=True) + self.eps)
        return Tensor((arr / rms) * self.weight.numpy(), x.device)


class LayerNorm(Module):
    """Standard LayerNorm (layers.py:52-67).  Not on the retention path:
    kept for API completeness on CPU tensors only."""

    def __init__(self, d_model: int, eps: float = 1e-5):
        super().__init__()
        self.d_model = d_model
        self.eps = eps
        self.weight = Parameter(Tensor(np.ones(d_model, dtype=np.float32)))
        self.bias = Parameter(Tensor(np.zeros(d_model, dtype=np.float32)))

    def forward(self, x: Tensor) -> Tensor:
        if x.device.is_cuda:
            raise NotImplementedError("LayerNorm is not part of the retention hot path (no CUDA kernel)")
        arr = x.numpy()
        mean = np.mean(arr, axis=-1, keepdims=True)
        var = np.var(arr, axis=-1, keepdims=True)
        return Tensor(((arr - mean) / np.sqrt(var + self.eps)) * self.weight.numpy() + self.bias.numpy(), x.device)


class SwiGLU(Module):
    """SwiGLU feed-forward network (layers.py:70-88): W_down(silu(W_gate x) * W_up x).

    On CUDA the gate and up weights are packed into one [2f, d] matrix (gate
    rows first, the layout of AceEngine's w_gate_up, cpu/swiglu.rs:7-8), so
    the pair is one GEMM followed by the fused SwiGLU kernel.
    """

    def __init__(self, d_model: int, hidden_dim: Optional[int] = None, multiple_of: int = 64):
        super().__init__()
        if hidden_dim is None:
            hidden_dim = int(2 * (4 * d_model) / 3)
            hidden_dim = multiple_of * ((hidden_dim + multiple_of - 1) // multiple_of)
        self.hidden_dim = hidden_dim
        self.w_gate = Linear(d_model, hidden_dim, bias=False)
        self.w_up = Linear(d_model, hidden_dim, bias=False)
        self.w_down = Linear(hidden_dim, d_model, bias=False)
        self._gate_up = None

    def _on_device(self) -> None:
        self._gate_up = None
        if self.w_gate.weight.device.is_cuda:
            import torch

            self._gate_up = torch.cat([self.w_gate.weight.torch, self.w_up.weight.torch], 0).contiguous()

    def forward(self, x: Tensor) -> Tensor:
        if x.device.is_cuda:
            ops = _cuda_ops()
            if self._gate_up is None:
                self._on_device()
            if self._gate_up is None:
                raise ValueError("SwiGLU weights are not on the input's CUDA device; call .to(device) first")
            gu = ops.linear(x.torch, self._gate_up)
            h = ops.swiglu_packed(gu)
            return Tensor._wrap(ops.linear(h, self.w_down.weight.torch), x.device)
        gate = self.w_gate(x).numpy()
        up = self.w_up(x).numpy()
        silu = gate / (1.0 + np.exp(-gate))
        return self.w_down(Tensor(silu * up, x.device))
