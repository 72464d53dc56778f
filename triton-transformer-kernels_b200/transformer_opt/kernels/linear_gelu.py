"""Block GEMMs with their elementwise consumers fused on sm_100a (libb200tk.so):
the FFN input projection with its exact GELU, and out_proj / ffn_out with the
residual add that follows them.

``fused_linear_gelu(x, weight, bias)`` computes
``F.gelu(F.linear(x, weight, bias), approximate="none")`` -- the
``F.gelu(layer.ffn_in(h))`` pair of the reference's block
(benchmarks/torch_transformer_benchmark.py:131, 141; placed by the fused layer
loop at transformer_opt/submission.py:506-508) -- as one tcgen05 GEMM whose
epilogue adds the bias and applies the GELU before the single store.

float32 inputs multiply as TF32 (what an fp32 Linear computes with
``torch.backends.cuda.matmul.allow_tf32``). The tensor cores read the top 19
bits of each operand (truncation); a TF32 cuBLAS matmul rounds to nearest, so
callers that must match it pass operands already rounded to TF32 (the model
rounds the weight once and has the preceding LayerNorm round x). float16 /
bfloat16 round the biased fp32 sum to the input dtype before the GELU, as the
unfused Linear's output tensor does. Unsupported calls raise ``ValueError``; a missing library
raises ``RuntimeError``. No fallback.
"""

from __future__ import annotations

from typing import Optional

import torch

from transformer_opt.config import SUPPORTED_DTYPES, device_supported
from transformer_opt.kernels import _native


def linear_gelu_unsupported_reason(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    *,
    x_planned: bool = False,
) -> Optional[str]:
    """Why ``fused_linear_gelu`` would reject these tensors, or None.

    With ``x_planned`` x stands for a fresh contiguous tensor of its shape,
    dtype and device (its own strides and address are not checked)."""
    if x.device.type != "cuda":
        return "fused linear GELU requires CUDA tensors"
    reason = device_supported(x.device)
    if reason is not None:
        return reason
    if x.dtype not in SUPPORTED_DTYPES:
        return "fused linear GELU supports float32, float16 and bfloat16"
    if x.ndim < 2:
        return "x must have rank two or higher"
    if weight.ndim != 2 or weight.shape[1] != x.shape[-1]:
        return "weight must be [out_features, in_features] with in_features == x.shape[-1]"
    if weight.dtype != x.dtype or weight.device != x.device:
        return "weight must match x's dtype and device"
    if bias is not None and (
        bias.shape != (weight.shape[0],) or bias.dtype != x.dtype or bias.device != x.device
    ):
        return "bias must be [out_features] with x's dtype and device"
    if (not x_planned and not x.is_contiguous()) or not weight.is_contiguous() or (
        bias is not None and not bias.is_contiguous()
    ):
        return "fused linear GELU requires contiguous tensors"
    elem = x.element_size()
    if (x.shape[-1] * elem) % 16 or (weight.shape[0] * elem) % 16:
        return "in_features and out_features must be multiples of 16 bytes of elements"
    for t in (None if x_planned else x, weight, bias):
        if t is not None and t.data_ptr() % 16:
            return "tensors must be 16-byte aligned"
    return None


def fused_linear_gelu(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``gelu(x @ weight.T + bias)`` (exact erf GELU) on the current stream."""
    reason = linear_gelu_unsupported_reason(x, weight, bias)
    if reason is not None:
        raise ValueError(reason)
    shape = (*x.shape[:-1], weight.shape[0])
    if out is None:
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
    elif out.shape != shape or out.dtype != x.dtype or out.device != x.device or (
        not out.is_contiguous() or out.data_ptr() % 16
    ):
        raise ValueError("out must be a contiguous, 16-byte aligned tensor of the output shape")
    if x.numel() == 0:
        return out
    _native.linear_gelu_fwd(x, weight, bias, out)
    return out


def fused_linear_residual(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    residual: torch.Tensor,
    valid_rows: Optional[torch.Tensor] = None,
    *,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``residual + F.linear(x, weight, bias)`` as one GEMM whose epilogue adds
    the residual (the projection rounded to x's dtype first, as the unfused
    Linear's output tensor is); rows where ``valid_rows`` is False are
    written as zeros. ``out`` may be ``residual`` itself (in place)."""
    reason = linear_gelu_unsupported_reason(x, weight, bias)
    if reason is not None:
        raise ValueError(reason)
    shape = (*x.shape[:-1], weight.shape[0])
    if residual.shape != shape or residual.dtype != x.dtype or residual.device != x.device or (
        not residual.is_contiguous() or residual.data_ptr() % 16
    ):
        raise ValueError("residual must be a contiguous, 16-byte aligned tensor of the output shape")
    if valid_rows is not None and (
        valid_rows.shape != shape[:-1] or valid_rows.dtype is not torch.bool
        or valid_rows.device != x.device or not valid_rows.is_contiguous()
    ):
        raise ValueError("valid_rows must be a contiguous bool tensor of the row shape on x's device")
    if out is None:
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
    elif out.shape != shape or out.dtype != x.dtype or out.device != x.device or (
        not out.is_contiguous() or out.data_ptr() % 16
    ):
        raise ValueError("out must be a contiguous, 16-byte aligned tensor of the output shape")
    if x.numel() == 0:
        return out
    _native.linear_residual_fwd(x, weight, bias, residual, valid_rows, out)
    return out
