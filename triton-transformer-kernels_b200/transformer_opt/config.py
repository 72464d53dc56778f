"""Support envelope of the sm_100a kernels.

Mirrors transformer_opt/config.py of the reference (ATTENTION_BACKENDS :11,
SUPPORTED_HEAD_DIMS :12, SUPPORTED_DTYPES :18, _validate_qkv_contract
:115-140, triton_attention_support :143-175) with the envelope of this
implementation: bfloat16 joins float16/float32, the sequence limit grows to
65536, and the device must be a B200-class GPU (compute capability 10.0),
the only architecture the library is compiled for.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

# "b200" is the sm_100a kernel route. "triton" is accepted as the
# reference's name for its custom-kernel route and maps to "b200".
ATTENTION_BACKENDS = ("auto", "b200", "triton", "sdpa", "reference")
CUSTOM_BACKEND = "b200"
LEGACY_CUSTOM_BACKEND = "triton"
SUPPORTED_HEAD_DIMS = frozenset({8, 16, 32, 64, 128})
SUPPORTED_DTYPES = frozenset({torch.float16, torch.bfloat16, torch.float32})
MIN_CUDA_CAPABILITY = (10, 0)
MAX_CUDA_CAPABILITY = (10, 0)
MAX_SEQUENCE_LENGTH = 65536
MAX_NORMALIZED_WIDTH = 65536


@dataclass(frozen=True)
class SupportResult:
    supported: bool
    reason: str


def _validate_qkv_contract(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor],
) -> Optional[str]:
    """The tensor contract of the attention entry point (reference :115-140)."""
    if q.ndim != 4:
        return "q, k, and v must have shape [batch, sequence, heads, head_dim]"
    if k.shape != q.shape or v.shape != q.shape:
        return "q, k, and v must have identical shapes"
    if k.dtype != q.dtype or v.dtype != q.dtype:
        return "q, k, and v must have identical dtypes"
    if k.device != q.device or v.device != q.device:
        return "q, k, and v must be on the same device"
    if q.shape[1] <= 0 or q.shape[2] <= 0 or q.shape[3] <= 0:
        return "sequence length, head count, and head dimension must be positive"
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        return "the head-dimension stride must be 1"
    if valid_token_mask is not None:
        if valid_token_mask.shape != q.shape[:2]:
            return "valid_token_mask must have shape [batch, sequence]"
        if valid_token_mask.dtype is not torch.bool:
            return "valid_token_mask must have dtype torch.bool"
        if valid_token_mask.device != q.device:
            return "valid_token_mask must be on the q/k/v device"
    return None


# Compute capability per CUDA device index (a device's capability never
# changes; the model asks on every layer, so the query is made once).
_CAPABILITY: dict = {}


def device_supported(device: torch.device) -> Optional[str]:
    """None when `device` can run the sm_100a kernels, else the reason."""
    if device.type != "cuda":
        return "custom attention requires CUDA tensors"
    if not torch.cuda.is_available():
        return "CUDA is unavailable"
    index = device.index if device.index is not None else torch.cuda.current_device()
    capability = _CAPABILITY.get(index)
    if capability is None:
        capability = torch.cuda.get_device_capability(index)
        _CAPABILITY[index] = capability
    if capability < MIN_CUDA_CAPABILITY or capability > MAX_CUDA_CAPABILITY:
        return (
            f"compute capability {capability} is not sm_100 "
            f"(the library is built for sm_100a only)"
        )
    return None


def b200_attention_support(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
) -> SupportResult:
    """Explain whether the sm_100a attention kernel can run these inputs."""
    contract_error = _validate_qkv_contract(q, k, v, valid_token_mask)
    if contract_error is not None:
        return SupportResult(False, contract_error)
    if q.device.type != "cuda":
        return SupportResult(False, "custom attention requires CUDA tensors")
    if q.dtype not in SUPPORTED_DTYPES:
        return SupportResult(False, "custom attention supports float16, bfloat16 and float32")
    if q.shape[-1] not in SUPPORTED_HEAD_DIMS:
        return SupportResult(
            False,
            f"head_dim={q.shape[-1]} is outside {sorted(SUPPORTED_HEAD_DIMS)}",
        )
    if q.shape[1] > MAX_SEQUENCE_LENGTH:
        return SupportResult(
            False,
            f"seq_len={q.shape[1]} exceeds the validated maximum {MAX_SEQUENCE_LENGTH}",
        )
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return SupportResult(False, "custom attention is forward-inference only")
    device_error = device_supported(q.device)
    if device_error is not None:
        return SupportResult(False, device_error)
    return SupportResult(True, "inside the validated sm_100a forward envelope")


# The reference's public name for the same query (transformer_opt/__init__.py).
triton_attention_support = b200_attention_support
