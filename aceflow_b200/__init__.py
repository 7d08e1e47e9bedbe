"""aceflow_b200 — B200-native (sm_100a) retention hot path for AceFlow.

Mirrors the reference package's retention API (``aceflow.Device``,
``aceflow.Tensor``, ``aceflow.nn``, ``aceflow.ops``) with a CUDA device kind
(``Device.cuda(i)``), backed by the C-ABI library ``libaceflow_cuda.so``
(include/aceflow_cuda.h).  ``import aceflow_b200 as af`` gives the same names
as ``import aceflow as af`` for the retention path.
"""
from .core.device import Device
from .core.tensor import Tensor
from . import nn
from . import ops

__version__ = "0.1.0"

__all__ = ["Device", "Tensor", "nn", "ops"]
