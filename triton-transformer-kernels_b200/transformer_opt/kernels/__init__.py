"""sm_100a kernels of the hot path (libb200tk.so through ctypes)."""

from .attention import attention_route, b200_attention, b200_available
from .linear_gelu import fused_linear_gelu, fused_linear_residual, linear_gelu_unsupported_reason
from .residual_layer_norm import fused_residual_layer_norm, layer_norm

__all__ = [
    "attention_route",
    "b200_attention",
    "b200_available",
    "fused_linear_gelu",
    "fused_linear_residual",
    "fused_residual_layer_norm",
    "layer_norm",
    "linear_gelu_unsupported_reason",
]
