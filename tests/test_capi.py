"""The C ABI (CPU): libb200tk.so loads without a GPU, exports every symbol
include/b200tk.h declares, and its host-side validation and routing behave
as documented. No kernel is launched here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from transformer_opt.kernels import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200tk.h"


def _declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"B200TK_API\s+[\w\s\*]+?\b(b200tk_\w+)\s*\(", text)


def test_library_loads_and_reports_abi_version():
    lib = _native.load()
    header_version = int(re.search(r"#define B200TK_ABI_VERSION (\d+)", HEADER.read_text()).group(1))
    assert lib.b200tk_abi_version() == header_version


def test_every_declared_symbol_is_exported():
    lib = _native.load()
    declared = _declared_symbols()
    assert len(declared) >= 7
    for name in declared:
        assert hasattr(lib, name), f"{name} is declared in b200tk.h but not exported"
    assert set(declared) == set(_native.SIGNATURES), "ctypes signatures out of sync with header"


def test_header_constants_match_binding():
    text = HEADER.read_text()

    def const(name):
        return int(re.search(rf"#define {name} \(?(-?\d+)u?\)?", text).group(1))

    assert const("B200TK_ERR_INVALID_ARGUMENT") == _native.ERR_INVALID_ARGUMENT
    assert const("B200TK_ERR_UNSUPPORTED") == _native.ERR_UNSUPPORTED
    assert const("B200TK_DTYPE_FLOAT32") == _native.DTYPE_CODES[torch.float32]
    assert const("B200TK_DTYPE_FLOAT16") == _native.DTYPE_CODES[torch.float16]
    assert const("B200TK_DTYPE_BFLOAT16") == _native.DTYPE_CODES[torch.bfloat16]
    assert const("B200TK_RLN_NO_UPDATE") == _native.RLN_NO_UPDATE
    assert const("B200TK_RLN_ROUND_TF32") == _native.RLN_ROUND_TF32
    assert const("B200TK_ROUTE_TCGEN05") == _native.ROUTE_TCGEN05


def _route(ptrs, strides, dtype=2, shape=(2, 128, 4, 64)):
    lib = _native.load()
    arrs = [(ctypes.c_int64 * 3)(*s) for s in strides]
    return lib.b200tk_attention_route(
        ctypes.c_void_p(ptrs[0]), arrs[0], ctypes.c_void_p(ptrs[1]), arrs[1],
        ctypes.c_void_p(ptrs[2]), arrs[2], dtype, *shape,
    )


def test_route_selects_tcgen05_for_aligned_views_and_generic_otherwise():
    b, s, h, d = 2, 128, 4, 64
    packed = (s * 3 * h * d, 3 * h * d, d)  # [B,S,3,H,D] packed-QKV view strides
    base = 1 << 20
    ptrs = (base, base + h * d * 2, base + 2 * h * d * 2)
    assert _route(ptrs, [packed] * 3) == _native.ROUTE_TCGEN05
    assert _route((base + 2, base, base), [packed] * 3) == _native.ROUTE_GENERIC  # misaligned q
    odd = (s * 3 * h * d, 3 * h * d + 1, d)  # seq stride not 16-byte multiple
    assert _route(ptrs, [odd, packed, packed]) == _native.ROUTE_GENERIC
    assert _route(ptrs, [packed] * 3, shape=(b, s, h, 32)) == _native.ROUTE_GENERIC


@pytest.mark.parametrize(
    "shape,dtype,code",
    [
        ((1, 16, 2, 48), 2, _native.ERR_UNSUPPORTED),  # head_dim outside the set
        ((1, 0, 2, 64), 2, _native.ERR_INVALID_ARGUMENT),  # empty sequence
        ((1, 16, 2, 64), 9, _native.ERR_INVALID_ARGUMENT),  # unknown dtype
    ],
)
def test_attention_validation_errors_need_no_gpu(shape, dtype, code):
    lib = _native.load()
    st = (ctypes.c_int64 * 3)(1, 1, 1)
    rc = lib.b200tk_attention_fwd(
        ctypes.c_void_p(16), st, ctypes.c_void_p(16), st, ctypes.c_void_p(16), st,
        None, None, ctypes.c_void_p(16), dtype, *shape, 0, 1.0, None,
    )
    assert rc == code
    assert lib.b200tk_last_error()


def test_residual_layer_norm_validation_errors_need_no_gpu():
    lib = _native.load()
    p = ctypes.c_void_p(16)
    rc = lib.b200tk_residual_layer_norm_fwd(p, p, p, None, None, p, p, 0, 4, 70000, 1e-5, 0, None)
    assert rc == _native.ERR_UNSUPPORTED
    rc = lib.b200tk_residual_layer_norm_fwd(p, p, p, None, None, p, p, 0, 4, 64, 1e-5, 1, None)
    assert rc == _native.ERR_INVALID_ARGUMENT  # zeroing without a mask
    assert b"mask" in lib.b200tk_last_error()
    rc = lib.b200tk_residual_layer_norm_fwd(p, p, p, None, None, p, p, 0, 0, 64, 1e-5, 0, None)
    assert rc == _native.OK  # zero rows: nothing to launch


def test_linear_gelu_validation_errors_need_no_gpu():
    lib = _native.load()
    p = ctypes.c_void_p(16)
    # in_features of 6 fp32 = 24 bytes: not a multiple of 16 bytes
    assert lib.b200tk_linear_gelu_fwd(p, p, None, p, 0, 4, 6, 32, None) == _native.ERR_UNSUPPORTED
    assert b"16 bytes" in lib.b200tk_last_error()
    # out_features of 12 bf16 = 24 bytes
    assert lib.b200tk_linear_gelu_fwd(p, p, None, p, 2, 4, 64, 12, None) == _native.ERR_UNSUPPORTED
    assert lib.b200tk_linear_gelu_fwd(p, p, None, p, 9, 4, 64, 64, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.b200tk_linear_gelu_fwd(p, p, None, p, 0, 4, 0, 64, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.b200tk_linear_gelu_fwd(p, p, None, p, 0, -1, 64, 64, None) == _native.ERR_INVALID_ARGUMENT
    # misaligned pointer
    odd = ctypes.c_void_p(24)
    assert lib.b200tk_linear_gelu_fwd(odd, p, None, p, 0, 4, 64, 64, None) == _native.ERR_UNSUPPORTED
    # zero rows: nothing to launch
    assert lib.b200tk_linear_gelu_fwd(p, p, None, p, 0, 0, 64, 64, None) == _native.OK


def test_residual_layer_norm_round_tf32_flag_validation_needs_no_gpu():
    lib = _native.load()
    p = ctypes.c_void_p(16)
    flag = _native.RLN_ROUND_TF32
    # TF32 rounding of the normalized output is defined for float32 only
    rc = lib.b200tk_residual_layer_norm_fwd(p, p, p, None, None, p, p, 2, 4, 64, 1e-5, flag, None)
    assert rc == _native.ERR_INVALID_ARGUMENT
    assert b"float32" in lib.b200tk_last_error()
    rc = lib.b200tk_residual_layer_norm_fwd(p, p, p, None, None, p, p, 0, 4, 64, 1e-5, 16, None)
    assert rc == _native.ERR_INVALID_ARGUMENT  # unknown flag bit
    rc = lib.b200tk_residual_layer_norm_fwd(p, p, p, None, None, p, p, 0, 0, 64, 1e-5, flag, None)
    assert rc == _native.OK  # float32 with the flag, zero rows: nothing to launch


def test_work_item_range_is_checked_before_any_launch():
    # bf16 head_dim 128: 256 query rows per item. S = 768 gives 3 tiles per
    # (batch, head); the causal pair schedule numbers 4 items per batch-head,
    # and 4 * 2^29 items overflow int while 3 * 2^29 do not: the shape must be
    # rejected by the host-side check, not launched with a wrapped count.
    s, h, d = 768, 512, 128
    contiguous = (s * h * d, h * d, d)
    base = 1 << 20
    ptrs = (base, base, base)
    assert _route(ptrs, [contiguous] * 3, shape=(1 << 20, s, h, d)) == _native.ERR_UNSUPPORTED
    assert b"work-item" in _native.load().b200tk_last_error()
    assert _route(ptrs, [contiguous] * 3, shape=(1 << 10, s, h, d)) == _native.ROUTE_TCGEN05
    # the CUDA-core route (head_dim 32: 128 rows per CTA, 6 per batch-head)
    narrow = (s * h * 32, h * 32, 32)
    assert _route(ptrs, [narrow] * 3, shape=(1 << 20, s, h, 32)) == _native.ERR_UNSUPPORTED
    assert _route(ptrs, [narrow] * 3, shape=(1 << 10, s, h, 32)) == _native.ROUTE_GENERIC


def test_attention_schedule_validation_needs_no_gpu():
    # An unknown schedule is an invalid argument; an explicit RESIDENT request
    # outside its envelope (head_dim 128, seq_len 513, float32, scale <= 0)
    # is refused before anything is launched.
    lib = _native.load()
    base = 1 << 20

    def call(schedule, dtype=2, shape=(2, 128, 4, 64), scale=0.125):
        b, s, h, d = shape
        st = (ctypes.c_int64 * 3)(s * h * d, h * d, d)
        p = ctypes.c_void_p(base)
        return lib.b200tk_attention_fwd_scheduled(p, st, p, st, p, st, None, None, p, dtype,
                                                  b, s, h, d, 0, scale, schedule, None)

    assert call(4) == _native.ERR_INVALID_ARGUMENT
    assert b"schedule" in lib.b200tk_last_error()
    for kwargs in ({"shape": (2, 128, 4, 128)}, {"shape": (2, 513, 4, 64)}, {"dtype": 0},
                   {"scale": -0.125}):
        assert call(_native.SCHEDULES["resident"], **kwargs) == _native.ERR_UNSUPPORTED
        assert b"resident schedule" in lib.b200tk_last_error()
    # zero batch: validated, nothing to launch
    assert call(_native.SCHEDULES["resident"], shape=(0, 128, 4, 64)) == _native.OK
