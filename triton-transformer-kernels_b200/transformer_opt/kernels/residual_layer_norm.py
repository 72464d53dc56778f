"""Fused residual add + LayerNorm on sm_100a, called through libb200tk.so.

Same contract as the reference's ``fused_residual_layer_norm``
(transformer_opt/kernels/residual_layer_norm.py:159-238), widened from
float32-only to float32 / float16 / bfloat16 I/O with fp32 statistics.
Unsupported calls raise ``ValueError``; a missing library raises
``RuntimeError``. No fallback.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from transformer_opt.config import MAX_NORMALIZED_WIDTH, SUPPORTED_DTYPES, device_supported
from transformer_opt.kernels import _native


def _check_affine(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> None:
    width = x.shape[-1]
    if weight is None:
        raise ValueError("fused residual LayerNorm requires an affine weight")
    if weight.shape != (width,) or weight.device != x.device or weight.dtype != x.dtype:
        raise ValueError("weight must match the normalized feature dimension")
    if not weight.is_contiguous():
        raise ValueError("weight must be contiguous")
    if bias is not None:
        if bias.shape != (width,) or bias.device != x.device or bias.dtype != x.dtype:
            raise ValueError("bias must match the normalized feature dimension")
        if not bias.is_contiguous():
            raise ValueError("bias must be contiguous")
    if width > MAX_NORMALIZED_WIDTH:
        raise ValueError("normalized feature dimension exceeds the fused kernel limit")


def _check_mask(x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> None:
    if valid_token_mask is None:
        return
    if valid_token_mask.shape != x.shape[:-1]:
        raise ValueError("valid_token_mask must match every non-feature dimension")
    if valid_token_mask.dtype is not torch.bool or valid_token_mask.device != x.device:
        raise ValueError("valid_token_mask must be a co-located bool tensor")
    if not valid_token_mask.is_contiguous():
        raise ValueError("valid_token_mask must be contiguous")


def _check_input(x: torch.Tensor) -> None:
    if x.ndim < 2:
        raise ValueError("x must have rank two or higher")
    if x.device.type != "cuda":
        raise ValueError("fused residual LayerNorm requires co-located CUDA tensors")
    reason = device_supported(x.device)
    if reason is not None:
        raise ValueError(reason)
    if x.dtype not in SUPPORTED_DTYPES:
        raise ValueError("fused residual LayerNorm supports float32, float16 and bfloat16")
    if not x.is_contiguous():
        raise ValueError("fused residual LayerNorm requires contiguous inputs")


def fused_residual_layer_norm(
    x: torch.Tensor,
    update: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    eps: float,
    valid_token_mask: Optional[torch.Tensor] = None,
    *,
    zero_invalid_residual: bool = False,
    zero_invalid_normalized: bool = False,
    round_normalized_tf32: bool = False,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Return ``(x + update, layer_norm(x + update))`` from one kernel.

    ``round_normalized_tf32`` (float32 only; not in the reference's
    signature) rounds the normalized output to the nearest TF32 value, the
    operand rounding of a TF32 matmul, for the fused FFN projection whose
    tensor cores read its input as stored.
    """
    if x.shape != update.shape or x.ndim < 2:
        raise ValueError("x and update must have the same rank-two-or-higher shape")
    if update.device != x.device:
        raise ValueError("fused residual LayerNorm requires co-located CUDA tensors")
    if update.dtype is not x.dtype:
        raise ValueError("x and update must share a dtype")
    _check_input(x)
    if not update.is_contiguous():
        raise ValueError("fused residual LayerNorm requires contiguous inputs")
    if torch.is_grad_enabled() and (x.requires_grad or update.requires_grad):
        raise ValueError("fused residual LayerNorm is forward-inference only")
    _check_affine(x, weight, bias)
    if (zero_invalid_residual or zero_invalid_normalized) and valid_token_mask is None:
        raise ValueError("invalid-row zeroing requires valid_token_mask")
    _check_mask(x, valid_token_mask)
    _native.load()
    residual_out = torch.empty_like(x)
    normalized_out = torch.empty_like(x)
    flags = 0
    if zero_invalid_residual:
        flags |= _native.RLN_ZERO_INVALID_RESIDUAL
    if zero_invalid_normalized:
        flags |= _native.RLN_ZERO_INVALID_NORMALIZED
    if round_normalized_tf32:
        if x.dtype != torch.float32:
            raise ValueError("TF32 rounding applies to float32 only")
        flags |= _native.RLN_ROUND_TF32
    if x.numel():
        with torch.cuda.device(x.device):
            _native.residual_layer_norm_fwd(
                x, update, weight, bias, valid_token_mask, residual_out, normalized_out,
                eps, flags,
            )
    return residual_out, normalized_out


def layer_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    eps: float,
    valid_token_mask: Optional[torch.Tensor] = None,
    *,
    zero_invalid_normalized: bool = False,
    round_normalized_tf32: bool = False,
) -> torch.Tensor:
    """Plain LayerNorm over the last dimension through the same kernel
    (optionally zeroing invalid rows, or rounding the output to TF32 for
    float32, as in ``fused_residual_layer_norm``)."""
    _check_input(x)
    if torch.is_grad_enabled() and x.requires_grad:
        raise ValueError("fused LayerNorm is forward-inference only")
    _check_affine(x, weight, bias)
    if zero_invalid_normalized and valid_token_mask is None:
        raise ValueError("invalid-row zeroing requires valid_token_mask")
    _check_mask(x, valid_token_mask)
    _native.load()
    out = torch.empty_like(x)
    flags = _native.RLN_NO_UPDATE
    if zero_invalid_normalized:
        flags |= _native.RLN_ZERO_INVALID_NORMALIZED
    if round_normalized_tf32:
        if x.dtype != torch.float32:
            raise ValueError("TF32 rounding applies to float32 only")
        flags |= _native.RLN_ROUND_TF32
    if x.numel():
        with torch.cuda.device(x.device):
            _native.residual_layer_norm_fwd(
                x, None, weight, bias, valid_token_mask, None, out, eps, flags
            )
    return out
