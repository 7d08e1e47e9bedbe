"""af.Device with a CUDA kind (mirrors aceflow/core/device.py:11-73).

The reference knows "cpu" and "wgpu"; this build adds "cuda" (``Device.cuda(i)``,
``"cuda:i"``).  The WebGPU kind belongs to the reference's graphics-API
backend, which is not part of this build; asking for it raises ValueError.
"""
from __future__ import annotations

from typing import Optional, Union


class Device:
    """Device abstraction (CPU or CUDA)."""

    def __init__(self, spec: Optional[Union[str, "Device"]] = None):
        if isinstance(spec, Device):
            self.type, self.index = spec.type, spec.index
            return
        if spec is None:
            self.type, self.index = "cpu", 0
            return
        if not isinstance(spec, str):
            # torch.device or anything with .type/.index
            kind = getattr(spec, "type", None)
            if kind is None:
                raise ValueError(f"unsupported device spec {spec!r}")
            spec = f"{kind}:{getattr(spec, 'index', 0) or 0}"
        if ":" in spec:
            kind, idx = spec.split(":", 1)
            self.type, self.index = kind.strip().lower(), int(idx.strip())
        else:
            self.type, self.index = spec.strip().lower(), 0
        if self.type in ("gpu", "wgpu", "webgpu"):
            raise ValueError("the WebGPU backend is not part of aceflow_b200; use Device.cuda()")
        if self.type not in ("cpu", "cuda"):
            raise ValueError(f"unknown device type {self.type!r}")

    @classmethod
    def cpu(cls) -> "Device":
        return cls("cpu")

    @classmethod
    def cuda(cls, index: int = 0) -> "Device":
        return cls(f"cuda:{index}")

    @property
    def is_cuda(self) -> bool:
        return self.type == "cuda"

    def torch_device(self):
        import torch

        return torch.device("cuda", self.index) if self.is_cuda else torch.device("cpu")

    def __repr__(self) -> str:
        return f"Device(type='{self.type}', index={self.index})"

    def __str__(self) -> str:
        return f"{self.type}:{self.index}"

    def __eq__(self, other: object) -> bool:
        if isinstance(other, Device):
            return self.type == other.type and self.index == other.index
        if isinstance(other, str):
            return str(self) == other or self.type == other
        return False

    def __hash__(self) -> int:
        return hash((self.type, self.index))
