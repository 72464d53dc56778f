"""Fused attention forward on sm_100a, called through libb200tk.so.

Strict wrapper in the role of the reference's ``triton_attention``
(transformer_opt/kernels/attention.py:268-360): validate, allocate the
contiguous ``[B, S, H, D]`` output, launch on the current CUDA stream.
Unsupported inputs raise; there is no fallback in this module.
"""

from __future__ import annotations

from typing import Optional

import torch

from transformer_opt.config import b200_attention_support, device_supported
from transformer_opt.kernels import _native


def b200_available(device: Optional[torch.device] = None) -> bool:
    """True when CUDA, an sm_100 device and the built library are all present."""
    if not torch.cuda.is_available():
        return False
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    if device_supported(dev) is not None:
        return False
    return _native.available()


def b200_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
    *,
    causal: bool = False,
    scale: Optional[float] = None,
    schedule: str = "auto",
) -> torch.Tensor:
    """Run the fused kernel and return a fresh contiguous ``[B, S, H, D]`` tensor.

    ``schedule`` ("auto", "two_pass", "one_pass", "resident") picks the
    softmax schedule of 16-bit inputs on the tensor-core route: two passes
    round the normalised probabilities to the input dtype (the explicit
    reference's rounding); one pass rounds them before normalisation and does
    half the exponentials and two thirds of the MMAs; "resident" (head_dim
    64, at most 512 keys) keeps whole score rows in tensor memory and rounds
    like two passes with the work of one. "auto" takes "resident" where it
    applies, one pass from 4096 keys, else two passes. fp32 has a single
    schedule."""
    support = b200_attention_support(q, k, v, valid_token_mask)
    if not support.supported:
        raise ValueError(f"unsupported b200 attention input: {support.reason}")
    _native.load()  # raises RuntimeError when the library is missing
    head_dim = q.shape[-1]
    softmax_scale = head_dim**-0.5 if scale is None else float(scale)
    output = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if output.numel() == 0:
        return output
    with torch.cuda.device(q.device):
        _native.attention_fwd(q, k, v, valid_token_mask, output, causal, softmax_scale, schedule)
    return output


def attention_route(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> str:
    """Name of the kernel the library picks: "tcgen05" or "generic"."""
    code = _native.attention_route(q, k, v)
    return "tcgen05" if code == _native.ROUTE_TCGEN05 else "generic"
