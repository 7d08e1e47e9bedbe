from .device import Device
from .tensor import Tensor

__all__ = ["Device", "Tensor"]
