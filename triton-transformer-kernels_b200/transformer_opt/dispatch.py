"""Attention dispatch with an auditable record of the route taken.

Same public surface as the reference's transformer_opt/dispatch.py:
``attention_forward(q, k, v, valid_token_mask=None, *, causal=False,
scale=None, backend="auto") -> (output, AttentionDispatch)`` (:99-161) and
the error contract: an unknown backend raises ``ValueError`` (:26-30); a
forced custom backend raises ``RuntimeError`` when the kernel library or an
sm_100 device is unavailable and ``ValueError`` when the inputs are outside
the envelope (:116-123).

Routes:
  * "b200" (also requested as "triton", the reference's name for its
    custom-kernel route): the sm_100a fused kernel in libb200tk.so.
  * "reference": explicit matmul / fp32 softmax / matmul, the semantics of
    the reference's ``_reference_attention`` (:69-96).
  * "sdpa": ``torch.nn.functional.scaled_dot_product_attention``, only when
    requested explicitly.
``auto`` selects "b200" for every CUDA input inside the envelope and fails
loudly if the library is missing there; inputs outside the envelope (CPU
tensors, autograd, another GPU architecture) run the explicit reference
math, and the record says why.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from transformer_opt.config import (
    ATTENTION_BACKENDS,
    CUSTOM_BACKEND,
    LEGACY_CUSTOM_BACKEND,
    b200_attention_support,
    device_supported,
)
from transformer_opt.kernels import _native
from transformer_opt.kernels.attention import b200_attention, b200_available


@dataclass(frozen=True)
class AttentionDispatch:
    requested: str
    selected: str
    reason: str


def _validate_backend(backend: str) -> None:
    if backend not in ATTENTION_BACKENDS:
        raise ValueError(
            f"attention backend must be one of {ATTENTION_BACKENDS}, got {backend!r}"
        )


def _sdpa_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    scale: Optional[float],
) -> torch.Tensor:
    """PyTorch SDPA on [B, H, S, D] views, causal and key masks combined."""
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    attention_mask = None
    use_is_causal = causal
    if valid_token_mask is not None:
        attention_mask = valid_token_mask[:, None, None, :]
        if causal:
            seq_len = q.shape[1]
            keep = torch.ones((seq_len, seq_len), dtype=torch.bool, device=q.device).tril()
            attention_mask = attention_mask & keep[None, None]
            use_is_causal = False
    output = F.scaled_dot_product_attention(
        qh, kh, vh, attn_mask=attention_mask, is_causal=use_is_causal, scale=scale
    )
    return output.transpose(1, 2).contiguous()


def _reference_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
    causal: bool,
    scale: Optional[float],
) -> torch.Tensor:
    """Explicit attention with the model's dtype boundaries.

    scores = q k^T in the input dtype, times the scale (rounded to the input
    dtype again), -inf for the causal future and invalid keys, softmax in
    fp32, probabilities cast back to the input dtype, then P v.
    """
    qh = q.transpose(1, 2).contiguous()
    kh = k.transpose(1, 2).contiguous()
    vh = v.transpose(1, 2).contiguous()
    scores = torch.matmul(qh, kh.transpose(-2, -1))
    scores = scores * (q.shape[-1] ** -0.5 if scale is None else scale)
    if causal:
        seq_len = q.shape[1]
        future = torch.ones((seq_len, seq_len), dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(future, float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probabilities = torch.softmax(scores.float(), dim=-1).to(dtype=q.dtype)
    output = torch.matmul(probabilities, vh)
    return output.transpose(1, 2).contiguous()


def attention_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
    *,
    causal: bool = False,
    scale: Optional[float] = None,
    backend: str = "auto",
    schedule: str = "auto",
) -> Tuple[torch.Tensor, AttentionDispatch]:
    """Execute attention and return both the output and the dispatch record.

    ``schedule`` (not in the reference's signature) picks the softmax
    schedule of 16-bit inputs on the custom route: "two_pass" rounds
    normalised probabilities (the explicit math's rounding), "one_pass" is
    the online softmax, "resident" rounds like "two_pass" with whole score
    rows held on chip (head_dim 64, at most 512 keys); "auto" takes
    "resident" where it applies, one pass from 4096 keys on, else two
    passes."""
    _validate_backend(backend)
    support = b200_attention_support(q, k, v, valid_token_mask)

    if backend in (CUSTOM_BACKEND, LEGACY_CUSTOM_BACKEND):
        if not b200_available(q.device if q.is_cuda else None):
            detail = device_supported(q.device) if q.is_cuda else "CUDA tensors are required"
            if detail is None:
                detail = _native.load_error() or "libb200tk.so could not be loaded"
            raise RuntimeError(f"custom attention was forced but is unavailable: {detail}")
        if not support.supported:
            raise ValueError(f"custom attention was forced but unsupported: {support.reason}")
        output = b200_attention(
            q, k, v, valid_token_mask, causal=causal, scale=scale, schedule=schedule
        )
        return output, AttentionDispatch(backend, CUSTOM_BACKEND, support.reason)

    if backend == "auto" and support.supported:
        # Inside the envelope the kernel is the only route: a missing library
        # is an error here, never a silent downgrade.
        output = b200_attention(
            q, k, v, valid_token_mask, causal=causal, scale=scale, schedule=schedule
        )
        return output, AttentionDispatch("auto", CUSTOM_BACKEND, support.reason)

    if backend == "sdpa":
        output = _sdpa_attention(q, k, v, valid_token_mask, causal, scale)
        return output, AttentionDispatch("sdpa", "sdpa", "explicit SDPA backend")

    reason = "explicit reference backend" if backend == "reference" else support.reason
    output = _reference_attention(q, k, v, valid_token_mask, causal, scale)
    return output, AttentionDispatch(backend, "reference", reason)
