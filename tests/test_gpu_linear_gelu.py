"""FFN input projection + exact GELU (libb200tk's tcgen05 GEMM with a GELU
epilogue) on a B200 against the oracle's ``linear_gelu``
(benchmarks/torch_transformer_benchmark.py:141).

Four kinds of check:
  * the epilogue alone: with an identity weight the GEMM is exact, so the
    output must equal ATen's GELU of (x + bias) -- rounded to the dtype first
    for 16-bit models, as the unfused Linear's output is -- bit for bit for
    fp32 (same erff, same evaluation order); for 16-bit (a polynomial erfc,
    |error| <= 1.5e-7) within one unit of the output format everywhere and
    bit for bit on nearly all of |v| <= 2, where both erf forms are accurate;
  * the GEMM against a float64 reference with a rigorous per-element error
    bound (TF32 truncation of both operands for fp32, fp32 accumulation,
    16-bit rounding of the Linear's output), on ragged rows, ragged K
    stages, ragged column tiles and a persistent multi-tile case;
  * fp32 against the unfused oracle (cuBLAS TF32 Linear + ATen GELU) with the
    harness rule, abs_err <= 1e-3 OR abs_err <= 1e-2 * |ref|;
  * fp32 with operands rounded to TF32 beforehand (what the model feeds it)
    against cuBLAS TF32 + ATen GELU within fp32 accumulation-order error.
"""

from __future__ import annotations

import pytest
import torch

from oracle import explicit as oracle
from transformer_opt.kernels import _native, fused_linear_gelu

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
GELU_SLOPE = 1.13  # max |d gelu / dv| (at v ~ 2.4) is 1.1289


@pytest.fixture(autouse=True, scope="module")
def _device_status_clean():
    _native.device_status(0, clear=True)
    yield
    assert _native.device_status(0) == 0, "a kernel recorded a pipeline timeout"


@pytest.fixture(autouse=True)
def _tf32_allowed():
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    yield
    torch.backends.cuda.matmul.allow_tf32 = saved


def _tf32_exact(t: torch.Tensor) -> torch.Tensor:
    """t with the low 13 mantissa bits cleared (exactly representable in TF32)."""
    return (t.contiguous().view(torch.int32) & ~0x1FFF).view(torch.float32)


def _inputs(rows, k, n, dtype, seed, bias=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, device="cuda", generator=g).to(dtype)
    bound = k ** -0.5  # nn.Linear's default init range
    w = ((torch.rand(n, k, device="cuda", generator=g) * 2 - 1) * bound).to(dtype)
    b = ((torch.rand(n, device="cuda", generator=g) * 2 - 1) * bound).to(dtype) if bias else None
    return x, w, b


def _check_against_fp64(out, x, w, b):
    """|out - gelu(x w^T + b)| within the error bound of this kernel's arithmetic."""
    k = x.shape[-1]
    x64, w64 = x.double(), w.double()
    lin = x64 @ w64.t() + (b.double() if b is not None else 0.0)
    ref = torch.nn.functional.gelu(lin)
    mag = x64.abs() @ w64.abs().t()  # sum_k |x_k w_k|
    acc = k * 2.0 ** -22  # fp32 accumulation
    # fp32 GELU: erf's absolute error (a few units of 2^-24 at |erf| ~ 1)
    # times v / 2, which dominates where 1 + erf cancels (v << 0)
    gelu_err = 2.0 ** -22 * lin.abs() + 2.0 ** -21 * ref.abs()
    if x.dtype == torch.float32:
        # TF32 truncation of both operands: < 2^-10 relative each
        lin_err = (2.0 ** -9 + 2.0 ** -19 + acc) * mag + 2.0 ** -23 * lin.abs()
        out_err = 0.0
    else:
        # half a unit in the last place, relative; fp16 also has subnormals
        # (absolute spacing 2^-24)
        unit = 2.0 ** -8 if x.dtype == torch.bfloat16 else 2.0 ** -11
        tiny = 2.0 ** -126 if x.dtype == torch.bfloat16 else 2.0 ** -25
        # the Linear's output is rounded to the dtype, and an accumulation
        # order different from the reference's may cross a rounding boundary
        lin_err = acc * mag + unit * lin.abs() + tiny
        out_err = unit * ref.abs() + tiny
    tol = GELU_SLOPE * lin_err + gelu_err + out_err + 1e-30
    err = (out.double() - ref).abs()
    bad = ~(err <= tol)
    assert torch.isfinite(out).all()
    assert not bad.any(), (
        f"{int(bad.sum())}/{bad.numel()} elements outside the bound; "
        f"worst excess {(err - tol).max().item():.3g}"
    )


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [256, 512])
def test_epilogue_is_bitwise_aten_gelu(dtype, n):
    rows = 300  # ragged last row tile
    g = torch.Generator(device="cuda").manual_seed(7)
    x = (torch.randn(rows, n, device="cuda", generator=g) * 3).to(dtype)
    if dtype == torch.float32:
        x = _tf32_exact(x)
    b = (torch.randn(n, device="cuda", generator=g)).to(dtype)
    eye = torch.eye(n, device="cuda", dtype=dtype)
    out = fused_linear_gelu(x, eye, b)
    lin = (x.float() + b.float()).to(dtype)  # the Linear's output tensor
    expect = torch.nn.functional.gelu(lin, approximate="none")
    if dtype == torch.float32:
        assert torch.equal(out, expect), (out - expect).abs().max().item()
        return
    # one unit of the 16-bit format at the value (2^-7 / 2^-10 relative bounds
    # it), plus 1e-6 absolute for the far negative tail, where ATen's
    # 1 + erf cancels and the polynomial's absolute error dominates
    unit = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    err = (out.float() - expect.float()).abs()
    assert (err <= unit * expect.float().abs() + 1e-6).all(), err.max().item()
    central = lin.float().abs() <= 2.0
    same = (out == expect)[central].float().mean().item()
    assert same > 0.99, same


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize(
    "rows,k,n",
    [
        (1, 64, 256),  # one row
        (127, 64, 256),  # one partial row tile
        (300, 200, 384),  # ragged rows, ragged last K stage, half column tile
        (129, 1024, 1040),  # ragged 32-column chunk at the right edge
        (2048, 1024, 4096),  # 512 tiles: persistent loop, ring and accumulator reuse
    ],
)
def test_matches_float64_within_bound(dtype, rows, k, n):
    x, w, b = _inputs(rows, k, n, dtype, seed=rows + k + n)
    out = fused_linear_gelu(x, w, b)
    assert out.shape == (rows, n) and out.dtype == dtype
    _check_against_fp64(out, x, w, b)


@pytest.mark.parametrize("dtype", DTYPES)
def test_without_bias_and_with_leading_dims(dtype):
    x, w, _ = _inputs(2 * 3 * 50, 128, 512, dtype, seed=3, bias=False)
    x3 = x.view(2, 3, 50, 128)
    out = fused_linear_gelu(x3, w, None)
    assert out.shape == (2, 3, 50, 512)
    _check_against_fp64(out.view(-1, 512), x, w, None)


@pytest.mark.parametrize("rows,k,n", [(4096, 1024, 4096), (512, 4096, 16384)])
def test_fp32_meets_the_harness_rule_against_the_unfused_oracle(rows, k, n):
    x, w, b = _inputs(rows, k, n, torch.float32, seed=11)
    out = fused_linear_gelu(x, w, b)
    ref = oracle.linear_gelu(x, w, b)  # cuBLAS TF32 Linear + ATen GELU
    err = (out - ref).abs()
    ok = (err <= 1e-3) | (err <= 1e-2 * ref.abs())
    assert ok.all(), f"failed={int((~ok).sum())} max_abs={err.max().item():.3g}"


def test_out_argument_and_repeated_calls_are_deterministic():
    x, w, b = _inputs(1000, 256, 768, torch.bfloat16, seed=5)
    out = torch.empty(1000, 768, device="cuda", dtype=torch.bfloat16)
    first = fused_linear_gelu(x, w, b, out=out).clone()
    second = fused_linear_gelu(x, w, b, out=out)
    assert second.data_ptr() == out.data_ptr()
    assert torch.equal(first, second)


def test_unsupported_shapes_raise_value_error():
    x = torch.randn(4, 6, device="cuda")  # 6 fp32 = 24 bytes: not a 16-byte multiple
    w = torch.randn(32, 6, device="cuda")
    with pytest.raises(ValueError):
        fused_linear_gelu(x, w, None)
    with pytest.raises(ValueError):
        fused_linear_gelu(x.cpu(), w.cpu(), None)


def _round_tf32(t: torch.Tensor) -> torch.Tensor:
    """Nearest TF32 values (ties away from zero), as fp32."""
    return ((t.contiguous().view(torch.int32) + 0x1000) & -0x2000).view(torch.float32)


@pytest.mark.parametrize("rows,k,n", [(4096, 1024, 4096), (1024, 4096, 16384)])
def test_fp32_with_tf32_rounded_operands_matches_cublas_tf32(rows, k, n):
    """With operands rounded to TF32 beforehand, every product is the one a
    TF32 cuBLAS matmul forms, so the fused result differs from cuBLAS TF32 +
    ATen GELU only by fp32 accumulation order (the model relies on this)."""
    x, w, b = _inputs(rows, k, n, torch.float32, seed=13)
    x, w = _round_tf32(x), _round_tf32(w)
    out = fused_linear_gelu(x, w, b)
    ref = oracle.linear_gelu(x, w, b)  # cuBLAS TF32 Linear + ATen GELU
    mag = x.abs() @ w.abs().t()
    tol = GELU_SLOPE * (k * 2.0 ** -22) * mag + 2.0 ** -21 * ref.abs() + 1e-7
    err = (out - ref).abs()
    assert (err <= tol).all(), f"worst excess {(err - tol).max().item():.3g}"
