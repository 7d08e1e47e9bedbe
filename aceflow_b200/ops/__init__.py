from .functional import gelu, matmul, rms_norm, silu, softmax, swiglu

__all__ = ["matmul", "rms_norm", "swiglu", "gelu", "silu", "softmax"]
