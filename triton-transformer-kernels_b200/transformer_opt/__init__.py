"""B200-native (sm_100a) kernels and dispatch for the Transformer inference
hot path: fused attention forward and fused residual-add + LayerNorm.

Public surface of the reference package of the same name
(transformer_opt/__init__.py): ``ATTENTION_BACKENDS``, ``AttentionDispatch``,
``attention_forward`` and the support query (``b200_attention_support``, also
exported under the reference's name ``triton_attention_support``).
"""

from .config import ATTENTION_BACKENDS, b200_attention_support, triton_attention_support
from .dispatch import AttentionDispatch, attention_forward

__all__ = [
    "ATTENTION_BACKENDS",
    "AttentionDispatch",
    "attention_forward",
    "b200_attention_support",
    "triton_attention_support",
]
