from .layers import LayerNorm, Linear, RMSNorm, SwiGLU
from .module import Module, Parameter
from .retention import MultiScaleRetention

__all__ = ["Module", "Parameter", "Linear", "RMSNorm", "LayerNorm", "SwiGLU", "MultiScaleRetention"]
