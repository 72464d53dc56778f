"""sm_100a kernels of the hot path (libb200tk.so through ctypes)."""

from .attention import attention_route, b200_attention, b200_available
from .residual_layer_norm import fused_residual_layer_norm, layer_norm

__all__ = [
    "attention_route",
    "b200_attention",
    "b200_available",
    "fused_residual_layer_norm",
    "layer_norm",
]
