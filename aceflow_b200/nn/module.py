"""Module / Parameter (mirrors aceflow/nn/module.py:7-68).

``Module.to(device)`` moves every Parameter, as the reference does
(module.py:57-62), and then calls ``_on_device()`` so a layer can pack its
weights for the device kernels (e.g. q/k/v fused into one [3d, d] matrix).
"""
from __future__ import annotations

from typing import Any, Dict, Iterator, Optional, Union

from ..core.device import Device
from ..core.tensor import Tensor


class Parameter(Tensor):
    """A Tensor that represents a learnable parameter in a Module."""

    __slots__ = ("requires_grad",)

    def __init__(self, data: Tensor, device=None):
        super().__init__(data, device)
        self.requires_grad = True


class Module:
    """Base class for all neural network modules."""

    def __init__(self) -> None:
        object.__setattr__(self, "_modules", {})
        object.__setattr__(self, "_parameters", {})
        self.training = True

    def register_parameter(self, name: str, param: Optional[Parameter]) -> None:
        if param is not None:
            self._parameters[name] = param
            object.__setattr__(self, name, param)

    def add_module(self, name: str, module: Optional["Module"]) -> None:
        if module is not None:
            self._modules[name] = module
            object.__setattr__(self, name, module)

    def __setattr__(self, name: str, value: Any) -> None:
        if isinstance(value, Parameter):
            self.__dict__.setdefault("_parameters", {})[name] = value
        elif isinstance(value, Module):
            self.__dict__.setdefault("_modules", {})[name] = value
        object.__setattr__(self, name, value)

    def parameters(self) -> Iterator[Parameter]:
        yield from self._parameters.values()
        for module in self._modules.values():
            yield from module.parameters()

    def named_parameters(self, prefix: str = ""):
        for n, p in self._parameters.items():
            yield prefix + n, p
        for mn, m in self._modules.items():
            yield from m.named_parameters(prefix + mn + ".")

    def train(self, mode: bool = True) -> "Module":
        self.training = mode
        for module in self._modules.values():
            module.train(mode)
        return self

    def eval(self) -> "Module":
        return self.train(False)

    @property
    def device(self) -> Device:
        for p in self.parameters():
            return p.device
        return Device("cpu")

    def to(self, device: Union[str, Device]) -> "Module":
        for name, param in list(self._parameters.items()):
            moved = Parameter(param.to(device))
            self._parameters[name] = moved
            object.__setattr__(self, name, moved)
        for module in self._modules.values():
            module.to(device)
        self._on_device()
        return self

    def cuda(self, index: int = 0) -> "Module":
        return self.to(Device.cuda(index))

    def _on_device(self) -> None:
        """Hook run after .to(): layers repack weights for their kernels."""

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        raise NotImplementedError

    def __call__(self, *args: Any, **kwargs: Any) -> Any:
        return self.forward(*args, **kwargs)
