"""ctypes binding of libb200tk.so, the C ABI declared in include/b200tk.h.

The library is built in-tree (``csrc/build.py``) and loaded from this
directory. Nothing here falls back to another implementation: if the library
is missing or fails to load, every entry point raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Optional, Sequence

import torch

LIB_NAME = "libb200tk.so"
LIB_PATH = Path(os.environ.get("B200TK_LIBRARY", Path(__file__).resolve().parent / LIB_NAME))

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

RLN_ZERO_INVALID_RESIDUAL = 1
RLN_ZERO_INVALID_NORMALIZED = 2
RLN_NO_UPDATE = 4
RLN_ROUND_TF32 = 8

STATUS_PIPELINE_TIMEOUT = 1
STATUS_SELFTEST_TIMEOUT = 2

SCHEDULES = {"auto": 0, "two_pass": 1, "one_pass": 2, "resident": 3}

ROUTE_TCGEN05 = 1
ROUTE_GENERIC = 2

# Every exported symbol and its ctypes signature (restype, argtypes).
_P = ctypes.c_void_p
_I64P = ctypes.POINTER(ctypes.c_int64)
_I64 = ctypes.c_int64
_I = ctypes.c_int
SIGNATURES = {
    "b200tk_abi_version": (_I, []),
    "b200tk_last_error": (ctypes.c_char_p, []),
    "b200tk_attention_fwd": (
        _I,
        [_P, _I64P, _P, _I64P, _P, _I64P, _P, _I64P, _P, _I, _I64, _I64, _I64, _I64, _I,
         ctypes.c_float, _P],
    ),
    "b200tk_attention_fwd_scheduled": (
        _I,
        [_P, _I64P, _P, _I64P, _P, _I64P, _P, _I64P, _P, _I, _I64, _I64, _I64, _I64, _I,
         ctypes.c_float, _I, _P],
    ),
    "b200tk_attention_route": (_I, [_P, _I64P, _P, _I64P, _P, _I64P, _I, _I64, _I64, _I64, _I64]),
    "b200tk_residual_layer_norm_fwd": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, ctypes.c_float, ctypes.c_uint32, _P],
    ),
    "b200tk_linear_gelu_fwd": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I64, _P]),
    "b200tk_linear_residual_fwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P]),
    "b200tk_device_status": (_I, [_I, ctypes.POINTER(ctypes.c_uint32), _I]),
    "b200tk_selftest_wait_timeout": (_I, [_I, ctypes.c_uint32, _P]),
}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise RuntimeError when unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            _load_error = (
                f"{LIB_NAME} is not built (expected at {LIB_PATH}); "
                "run csrc/build.py or __graft_entry__.build()"
            )
            raise RuntimeError(_load_error)
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            _load_error = f"failed to load {LIB_PATH}: {exc}"
            raise RuntimeError(_load_error) from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def load_error() -> Optional[str]:
    return _load_error


class NativeError(RuntimeError):
    """A libb200tk call returned an error code."""

    def __init__(self, code: int, message: str) -> None:
        super().__init__(f"libb200tk error {code}: {message}")
        self.code = code


def _check(rc: int) -> int:
    if rc < 0:
        msg = load().b200tk_last_error()
        text = msg.decode() if msg else "unknown error"
        if rc in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED):
            raise ValueError(text)
        raise NativeError(rc, text)
    return rc


def _strides(values: Sequence[int]):
    arr = (ctypes.c_int64 * len(values))(*values)
    return arr


def _stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def attention_fwd(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    mask: Optional[torch.Tensor],
    out: torch.Tensor,
    causal: bool,
    scale: float,
    schedule: str = "auto",
) -> None:
    """Launch fused attention on the current stream of q's device.

    ``schedule`` picks the 16-bit softmax schedule ("auto", "two_pass",
    "one_pass", "resident"; see B200TK_SCHEDULE_* in include/b200tk.h)."""
    lib = load()
    b, s, h, d = q.shape
    qs, ks, vs = _strides(q.stride()[:3]), _strides(k.stride()[:3]), _strides(v.stride()[:3])
    mptr, ms = None, None
    if mask is not None:
        mptr = ctypes.c_void_p(mask.data_ptr())
        ms = _strides(mask.stride())
    if schedule not in SCHEDULES:
        raise ValueError(f"schedule must be one of {tuple(SCHEDULES)}, got {schedule!r}")
    rc = lib.b200tk_attention_fwd_scheduled(
        ctypes.c_void_p(q.data_ptr()), qs,
        ctypes.c_void_p(k.data_ptr()), ks,
        ctypes.c_void_p(v.data_ptr()), vs,
        mptr, ms,
        ctypes.c_void_p(out.data_ptr()),
        DTYPE_CODES[q.dtype], b, s, h, d,
        1 if causal else 0, float(scale), SCHEDULES[schedule],
        _stream_handle(q.device),
    )
    _check(rc)


def attention_route(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> int:
    """Which kernel (ROUTE_TCGEN05 / ROUTE_GENERIC) attention_fwd would launch."""
    lib = load()
    b, s, h, d = q.shape
    rc = lib.b200tk_attention_route(
        ctypes.c_void_p(q.data_ptr()), _strides(q.stride()[:3]),
        ctypes.c_void_p(k.data_ptr()), _strides(k.stride()[:3]),
        ctypes.c_void_p(v.data_ptr()), _strides(v.stride()[:3]),
        DTYPE_CODES[q.dtype], b, s, h, d,
    )
    return _check(rc)


def residual_layer_norm_fwd(
    x: torch.Tensor,
    update: Optional[torch.Tensor],
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    mask: Optional[torch.Tensor],
    residual_out: Optional[torch.Tensor],
    normalized_out: torch.Tensor,
    eps: float,
    flags: int,
) -> None:
    """Launch fused residual + LayerNorm on the current stream of x's device."""
    lib = load()
    width = x.shape[-1]
    rows = x.numel() // width if width else 0

    def ptr(t: Optional[torch.Tensor]):
        return None if t is None else ctypes.c_void_p(t.data_ptr())

    rc = lib.b200tk_residual_layer_norm_fwd(
        ptr(x), ptr(update), ptr(weight), ptr(bias), ptr(mask),
        ptr(residual_out), ptr(normalized_out),
        DTYPE_CODES[x.dtype], rows, width, float(eps), int(flags),
        _stream_handle(x.device),
    )
    _check(rc)


def linear_gelu_fwd(
    x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], out: torch.Tensor
) -> None:
    """Launch out = gelu(x @ weight.T + bias) on the current stream of x's device."""
    lib = load()
    in_features = x.shape[-1]
    rows = x.numel() // in_features if in_features else 0
    rc = lib.b200tk_linear_gelu_fwd(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(weight.data_ptr()),
        None if bias is None else ctypes.c_void_p(bias.data_ptr()),
        ctypes.c_void_p(out.data_ptr()),
        DTYPE_CODES[x.dtype], rows, in_features, weight.shape[0],
        _stream_handle(x.device),
    )
    _check(rc)


def linear_residual_fwd(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    residual: torch.Tensor,
    valid_rows: Optional[torch.Tensor],
    out: torch.Tensor,
) -> None:
    """Launch out = residual + (x @ weight.T + bias) (rows zeroed where
    valid_rows is False) on the current stream of x's device."""
    lib = load()
    in_features = x.shape[-1]
    rows = x.numel() // in_features if in_features else 0
    rc = lib.b200tk_linear_residual_fwd(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(weight.data_ptr()),
        None if bias is None else ctypes.c_void_p(bias.data_ptr()),
        ctypes.c_void_p(residual.data_ptr()),
        None if valid_rows is None else ctypes.c_void_p(valid_rows.data_ptr()),
        ctypes.c_void_p(out.data_ptr()),
        DTYPE_CODES[x.dtype], rows, in_features, weight.shape[0],
        _stream_handle(x.device),
    )
    _check(rc)


def device_status(device: int = 0, clear: bool = False) -> int:
    """Synchronise `device` and read its status word (STATUS_* bits)."""
    lib = load()
    value = ctypes.c_uint32(0)
    _check(lib.b200tk_device_status(int(device), ctypes.byref(value), 1 if clear else 0))
    return int(value.value)


def selftest_wait_timeout(device: int = 0, timeout_us: int = 1000) -> None:
    """Run the bounded-wait self test on `device` (see include/b200tk.h)."""
    lib = load()
    with torch.cuda.device(device):
        stream = _stream_handle(torch.device("cuda", device))
        _check(lib.b200tk_selftest_wait_timeout(int(device), int(timeout_us), stream))


def abi_version() -> int:
    return int(load().b200tk_abi_version())
