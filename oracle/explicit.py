"""Explicit-math oracle for the Transformer inference hot path.

TEST INFRASTRUCTURE ONLY: the checker for libb200tk's kernels and for
UserOptimizedTransformer, and the timed CPU baseline. It is never called on
the product path.

Restates, with plain PyTorch ops (CPU or GPU), the reference project's
explicit model and per-op semantics:
  * model   : benchmarks/torch_transformer_benchmark.py:29-172
              (TransformerConfig, BaselineSelfAttention,
              BaselineTransformerBlock, BaselineTransformer) -- pre-LN blocks,
              fp32 softmax, padded rows zeroed.
  * harness : copy_model_weights :203-213, generate_random_case :234-272
              (and the no-mask variant of transformer_opt/submission.py:56-75),
              compare_outputs :289-356 (the exact OR rule
              abs_err <= atol OR abs_err <= rtol * |ref|, not isclose).
  * per-op  : reference_attention = transformer_opt/dispatch.py:69-96;
              residual_layer_norm = tests/test_gpu_residual_layer_norm.py:44-61
              (x + update, optional invalid-row zeroing, F.layer_norm);
              linear_gelu = the block's FFN input projection + exact GELU,
              benchmarks/torch_transformer_benchmark.py:141.
Parity is pinned by tests/test_oracle_golden.py against golden vectors that
tests/golden/make_golden.py produced by running the reference itself.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

ATOL = 1e-3  # the harness's per-element tolerance (README, north star)
RTOL = 1e-2


@dataclass(frozen=True)
class TransformerConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool


def _causal_future(seq_len: int, device) -> torch.Tensor:
    return torch.ones((seq_len, seq_len), dtype=torch.bool, device=device).triu(diagonal=1)


class BaselineSelfAttention(nn.Module):
    """Explicit multi-head self-attention (reference :59-122)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def _heads(self, t: torch.Tensor) -> torch.Tensor:
        b, s, _ = t.shape
        return t.view(b, s, self.num_heads, self.head_dim).transpose(1, 2).contiguous()

    def forward(self, x, valid_token_mask=None, causal=False):
        b, s, _ = x.shape
        q, k, v = self._heads(self.q_proj(x)), self._heads(self.k_proj(x)), self._heads(self.v_proj(x))
        scores = torch.matmul(q, k.transpose(-2, -1)) * self.scale
        if causal:
            scores = scores.masked_fill(_causal_future(s, x.device), float("-inf"))
        if valid_token_mask is not None:
            scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
        context = torch.matmul(probs, v).transpose(1, 2).contiguous().view(b, s, self.d_model)
        out = self.out_proj(context)
        if valid_token_mask is not None:
            out = out.masked_fill(~valid_token_mask[..., None], 0)
        return out


class BaselineTransformerBlock(nn.Module):
    """Pre-LN block (reference :125-145)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = BaselineSelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x, valid_token_mask, causal):
        x = x + self.attention(self.norm1(x), valid_token_mask, causal)
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


class BaselineTransformer(nn.Module):
    """Layer stack + final LayerNorm (reference :148-172)."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [
                BaselineTransformerBlock(config.d_model, config.num_heads, config.ffn_dim)
                for _ in range(config.num_layers)
            ]
        )
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x, valid_token_mask=None):
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        x = self.final_norm(x)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def copy_model_weights(baseline: nn.Module, optimized: nn.Module, strict: bool = True) -> None:
    """Load the baseline's parameters into the optimized model (reference :203-213)."""
    optimized.load_state_dict(copy.deepcopy(baseline.state_dict()), strict=strict)


def generate_random_case(
    config: TransformerConfig,
    device: torch.device,
    dtype: torch.dtype,
    seed: int,
    padding_ratio: float = 0.0,
    input_scale: float = 1.0,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """x ~ N(0,1) * input_scale from a seeded generator; prefix-valid padding.

    No padding returns ``valid_token_mask=None`` (the optimized path's
    contract, transformer_opt/submission.py:56-75).
    """
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    x = torch.randn(
        config.batch_size, config.seq_len, config.d_model,
        generator=generator, device=device, dtype=dtype,
    ) * input_scale
    if padding_ratio <= 0:
        return x, None
    min_valid = max(1, int(round(config.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(
        low=min_valid, high=config.seq_len + 1, size=(config.batch_size,),
        generator=generator, device=device,
    )
    mask = torch.arange(config.seq_len, device=device)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float


def compare_outputs(
    reference: torch.Tensor, optimized: torch.Tensor, rtol: float = RTOL, atol: float = ATOL
) -> AccuracyResult:
    """Per-element OR rule of the harness (reference :289-356)."""
    if reference.shape != optimized.shape:
        raise AssertionError(f"shape mismatch: {tuple(reference.shape)} vs {tuple(optimized.shape)}")
    ref = reference.detach().float()
    opt = optimized.detach().float()
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    err = (opt - ref).abs()
    passed = finite & ((err <= atol) | (err <= rtol * ref.abs()))
    failed = int((~passed).sum().item())
    flat = int(err.reshape(-1).argmax().item()) if err.numel() else 0
    index = []
    for size in reversed(reference.shape):
        index.append(flat % size)
        flat //= size
    worst = tuple(reversed(index))
    rel = err / ref.abs().clamp_min(1e-12)
    return AccuracyResult(
        passed=failed == 0,
        total_elements=reference.numel(),
        failed_elements=failed,
        max_abs_error=float(err.max().item()) if err.numel() else 0.0,
        max_relative_error=float(rel.max().item()) if rel.numel() else 0.0,
        mean_abs_error=float(err.mean().item()) if err.numel() else 0.0,
        worst_index=worst,
        reference_at_worst=float(ref[worst].item()) if err.numel() else 0.0,
        optimized_at_worst=float(opt[worst].item()) if err.numel() else 0.0,
    )


def reference_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
    causal: bool = False,
    scale: Optional[float] = None,
) -> torch.Tensor:
    """Explicit attention on [B, S, H, D] (transformer_opt/dispatch.py:69-96)."""
    qh, kh, vh = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    scores = torch.matmul(qh, kh.transpose(-2, -1))
    scores = scores * (q.shape[-1] ** -0.5 if scale is None else scale)
    if causal:
        scores = scores.masked_fill(_causal_future(q.shape[1], q.device), float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=q.dtype)
    return torch.matmul(probs, vh).transpose(1, 2).contiguous()


def reference_attention_rows(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    rows: Sequence[int],
    valid_token_mask: Optional[torch.Tensor] = None,
    causal: bool = False,
    scale: Optional[float] = None,
) -> torch.Tensor:
    """reference_attention restricted to query positions `rows` -> [B, len(rows), H, D].

    Query rows are independent in attention, so this equals
    ``reference_attention(...)[:, rows]`` at a fraction of the cost; it is how
    full-size shapes (S = 16384) are checked.
    """
    idx = torch.as_tensor(list(rows), device=q.device, dtype=torch.long)
    qh = q[:, idx].transpose(1, 2).contiguous()
    kh, vh = k.transpose(1, 2).contiguous(), v.transpose(1, 2).contiguous()
    scores = torch.matmul(qh, kh.transpose(-2, -1))
    scores = scores * (q.shape[-1] ** -0.5 if scale is None else scale)
    if causal:
        keys = torch.arange(q.shape[1], device=q.device)
        scores = scores.masked_fill(keys[None, :] > idx[:, None], float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=q.dtype)
    return torch.matmul(probs, vh).transpose(1, 2).contiguous()


def residual_layer_norm(
    x: torch.Tensor,
    update: Optional[torch.Tensor],
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    eps: float,
    valid_token_mask: Optional[torch.Tensor] = None,
    zero_invalid_residual: bool = False,
    zero_invalid_normalized: bool = False,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """(x + update, layer_norm(x + update)) with optional invalid-row zeroing.

    The residual is formed in the input dtype (as the model's ``x + y``
    does); the statistics come from F.layer_norm on it.
    """
    residual = x if update is None else x + update
    if zero_invalid_residual:
        residual = residual.masked_fill(~valid_token_mask[..., None], 0)
    normalized = F.layer_norm(residual, (x.shape[-1],), weight, bias, eps)
    if zero_invalid_normalized:
        normalized = normalized.masked_fill(~valid_token_mask[..., None], 0)
    return residual, normalized


def linear_gelu(
    x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]
) -> torch.Tensor:
    """The block's FFN input projection and activation,
    ``F.gelu(ffn_in(h), approximate="none")``
    (benchmarks/torch_transformer_benchmark.py:141): a Linear whose output is
    a tensor of x's dtype, then the exact (erf) GELU of that tensor."""
    return F.gelu(F.linear(x, weight, bias), approximate="none")



def baseline_forward_rows(
    model: BaselineTransformer,
    x: torch.Tensor,
    rows: Sequence[int],
    valid_token_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """BaselineTransformer(x)[:, rows] for a one-layer model, computing only `rows`.

    Every op except attention is row-local and attention rows are independent
    given all keys/values, so the result equals the full forward restricted
    to `rows`. Used to check shapes whose full explicit forward would not fit
    (S = 16384).
    """
    if len(model.layers) != 1:
        raise ValueError("row-restricted forward is defined for one-layer models")
    layer = model.layers[0]
    attn = layer.attention
    idx = torch.as_tensor(list(rows), device=x.device, dtype=torch.long)
    h = layer.norm1(x)
    b, s, _ = x.shape
    split = lambda t: t.view(b, t.shape[1], attn.num_heads, attn.head_dim)  # noqa: E731
    q = split(attn.q_proj(h[:, idx]))
    k, v = split(attn.k_proj(h)), split(attn.v_proj(h))
    # attention of the selected query positions against every key
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    scores = torch.matmul(qh, kh.transpose(-2, -1)) * attn.scale
    if model.config.causal:
        keys = torch.arange(s, device=x.device)
        scores = scores.masked_fill(keys[None, :] > idx[:, None], float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
    context = torch.matmul(probs, vh).transpose(1, 2).contiguous().view(b, len(idx), attn.d_model)
    attn_out = attn.out_proj(context)
    row_mask = None if valid_token_mask is None else valid_token_mask[:, idx]
    if row_mask is not None:
        attn_out = attn_out.masked_fill(~row_mask[..., None], 0)
    y = x[:, idx] + attn_out
    y = y + layer.ffn_out(F.gelu(layer.ffn_in(layer.norm2(y)), approximate="none"))
    if row_mask is not None:
        y = y.masked_fill(~row_mask[..., None], 0)
    y = model.final_norm(y)
    if row_mask is not None:
        y = y.masked_fill(~row_mask[..., None], 0)
    return y
