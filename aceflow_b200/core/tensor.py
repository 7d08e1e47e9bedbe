"""af.Tensor backed by torch storage (mirrors aceflow/core/tensor.py:14-118).

A Tensor lives on a CPU or a CUDA device.  Storage is a torch tensor in both
cases (torch is the device-memory allocator here, not the compute engine).
Arithmetic on a CUDA tensor goes through libaceflow_cuda.so; a CPU tensor
keeps the reference's numpy semantics.  Unlike the reference, constructing a
Tensor from a Tensor keeps its data on every device, so ``Parameter(Tensor)``
works without the compiled extension (the reference loses the numpy buffer,
aceflow/core/tensor.py:18-21 with aceflow/nn/module.py:10-12).

Extension over the reference: an optional ``dtype`` ("float32" or
"bfloat16"; bfloat16 only on CUDA) selecting the tensor-core prefill path.
"""
from __future__ import annotations

from typing import Any, List, Optional, Union

import numpy as np
import torch

from .device import Device

_DTYPES = {"float32": torch.float32, "fp32": torch.float32, "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
           torch.float32: torch.float32, torch.bfloat16: torch.bfloat16}


def _torch_dtype(dtype) -> torch.dtype:
    if dtype is None:
        return torch.float32
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype!r} (float32 or bfloat16)") from None


class Tensor:
    """Tensor on a CPU or CUDA device."""

    __slots__ = ("_t", "_device")

    def __init__(self, data: Union[np.ndarray, List[Any], "Tensor", torch.Tensor],
                 device: Optional[Union[Device, str]] = None, dtype=None):
        if isinstance(data, Tensor):
            self._t = data._t
            self._device = data._device
            if device is not None and Device(device) != self._device:
                moved = data.to(device)
                self._t, self._device = moved._t, moved._device
            if dtype is not None:
                self._t = self._t.to(_torch_dtype(dtype))
            return
        dev = Device(device)
        tdt = _torch_dtype(dtype)
        if tdt == torch.bfloat16 and not dev.is_cuda:
            raise ValueError("bfloat16 tensors are CUDA-only")
        if isinstance(data, torch.Tensor):
            t = data.detach()
        else:
            arr = np.asarray(data)
            if arr.dtype != np.float32:
                arr = arr.astype(np.float32)
            t = torch.from_numpy(np.ascontiguousarray(arr))
        self._t = t.to(device=dev.torch_device(), dtype=tdt).contiguous()
        self._device = dev

    # ---- wrappers -----------------------------------------------------------
    @classmethod
    def _wrap(cls, t: torch.Tensor, device: Device) -> "Tensor":
        res = cls.__new__(cls)
        res._t = t
        res._device = device
        return res

    @property
    def torch(self) -> torch.Tensor:
        """The underlying torch storage (same device, no copy)."""
        return self._t

    @property
    def shape(self) -> List[int]:
        return list(self._t.shape)

    @property
    def device(self) -> Device:
        return self._device

    @property
    def dtype(self) -> str:
        return "bfloat16" if self._t.dtype == torch.bfloat16 else "float32"

    def to(self, device: Optional[Union[Device, str]] = None, dtype=None) -> "Tensor":
        dev = self._device if device is None else Device(device)
        tdt = self._t.dtype if dtype is None else _torch_dtype(dtype)
        if tdt == torch.bfloat16 and not dev.is_cuda:
            raise ValueError("bfloat16 tensors are CUDA-only")
        return Tensor._wrap(self._t.to(device=dev.torch_device(), dtype=tdt).contiguous(), dev)

    def cuda(self, index: int = 0) -> "Tensor":
        return self.to(Device.cuda(index))

    def numpy(self) -> np.ndarray:
        t = self._t
        if t.dtype != torch.float32:
            t = t.float()
        return t.cpu().numpy() if t.is_cuda else t.numpy()

    # ---- constructors -------------------------------------------------------
    @classmethod
    def zeros(cls, shape: List[int], device: Optional[Union[Device, str]] = None, dtype=None) -> "Tensor":
        dev = Device(device)
        return cls._wrap(torch.zeros(shape, dtype=_torch_dtype(dtype), device=dev.torch_device()), dev)

    @classmethod
    def ones(cls, shape: List[int], device: Optional[Union[Device, str]] = None, dtype=None) -> "Tensor":
        dev = Device(device)
        return cls._wrap(torch.ones(shape, dtype=_torch_dtype(dtype), device=dev.torch_device()), dev)

    # ---- arithmetic ---------------------------------------------------------
    def matmul(self, other: "Tensor") -> "Tensor":
        """self [..., K] @ other [K, N] (aceflow/core/tensor.py:90-97)."""
        if self._device.is_cuda:
            from .. import cuda_ops

            if other._device != self._device:
                raise ValueError("matmul operands are on different devices")
            if len(other.shape) != 2:
                raise ValueError("matmul: right operand must be 2-D [K, N]")
            # the GEMM takes W as [N, K]; a transposed copy, as Linear.forward
            # makes in the reference (aceflow/nn/layers.py:30)
            w = other._t.t().contiguous()
            return Tensor._wrap(cuda_ops.linear(self._t.contiguous(), w), self._device)
        return Tensor(np.matmul(self.numpy(), other.numpy()), self._device)

    def __matmul__(self, other: "Tensor") -> "Tensor":
        return self.matmul(other)

    def __add__(self, other: Union["Tensor", float]) -> "Tensor":
        if self._device.is_cuda:
            from .. import cuda_ops

            if isinstance(other, Tensor):
                return Tensor._wrap(cuda_ops.add(self._t, other._t), self._device)
            return Tensor._wrap(cuda_ops.add_scalar(self._t, float(other)), self._device)
        arr = other.numpy() if isinstance(other, Tensor) else other
        return Tensor(self.numpy() + arr, self._device)

    def __repr__(self) -> str:
        return f"af.Tensor(shape={self.shape}, device='{self.device}', dtype={self.dtype})"
