"""Module structure of the Transformer whose inference forward this package
accelerates.

The parameter layout is the contract: attribute names and nesting equal those
of the organizer benchmark's ``BaselineTransformer``
(benchmarks/torch_transformer_benchmark.py:59-172 in the reference project),
so ``load_state_dict(baseline.state_dict(), strict=True)`` works in both
directions. Submodules are created in the same order, so the same
``torch.manual_seed`` yields the same default initialisation.

The model is pre-LayerNorm (:140-141): ``x = x + attn(norm1(x));
x = x + ffn(norm2(x))`` per block, padded rows zeroed after each block, then
``final_norm`` (:167-172). ``explicit_forward`` is that computation with
PyTorch ops; it serves inputs outside the fused kernels' envelope (CPU,
autograd).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class TransformerConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by num_heads ({self.num_heads})"
            )


class SelfAttentionWeights(nn.Module):
    """q/k/v/out projections of one attention layer (names fixed by the contract)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)


class TransformerBlockWeights(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = SelfAttentionWeights(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)


class TransformerWeights(nn.Module):
    """The full parameter tree: ``layers.{i}.*`` and ``final_norm``."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [
                TransformerBlockWeights(config.d_model, config.num_heads, config.ffn_dim)
                for _ in range(config.num_layers)
            ]
        )
        self.final_norm = nn.LayerNorm(config.d_model)


def split_heads(t: torch.Tensor, num_heads: int) -> torch.Tensor:
    """[B, S, d] -> [B, S, H, D] view."""
    b, s, d = t.shape
    return t.view(b, s, num_heads, d // num_heads)


def explicit_block(
    layer: TransformerBlockWeights,
    x: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    attention,
) -> torch.Tensor:
    """One pre-LN block with PyTorch ops; ``attention(layer.attention, h)`` returns [B,S,d]."""
    attn_out = attention(layer.attention, layer.norm1(x))
    if valid_token_mask is not None:
        attn_out = attn_out.masked_fill(~valid_token_mask[..., None], 0)
    x = x + attn_out
    x = x + layer.ffn_out(F.gelu(layer.ffn_in(layer.norm2(x)), approximate="none"))
    if valid_token_mask is not None:
        x = x.masked_fill(~valid_token_mask[..., None], 0)
    return x
