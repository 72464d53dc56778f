"""out_proj / ffn_out with the residual add fused (libb200tk's tcgen05 GEMM
with a residual epilogue) on a B200, against the unfused computation of the
reference's block, ``x + linear(h)`` (benchmarks/torch_transformer_benchmark.py
:140-141; the fused layer loop's residual points, transformer_opt/
submission.py:499-523).

  * the epilogue alone: with an identity weight the GEMM is exact, so the
    output must equal ATen's ``res + (x + bias)`` in the model dtype bit for
    bit (the projection rounded to the dtype before the add, as the unfused
    Linear's output tensor is);
  * the GEMM against a float64 reference within a rigorous per-element bound
    (16-bit: two roundings of the output format plus fp32 accumulation; fp32:
    TF32 truncation of both operands), on ragged rows, columns and K;
  * row zeroing by the valid-row mask, and in-place use (out = residual).
"""

from __future__ import annotations

import pytest
import torch

from transformer_opt.kernels import _native, fused_linear_residual

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
UNIT = {torch.float32: 2.0 ** -10, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


@pytest.fixture(autouse=True, scope="module")
def _device_status_clean():
    _native.device_status(0, clear=True)
    yield
    assert _native.device_status(0) == 0, "a kernel recorded a pipeline timeout"


def _tf32_exact(t):
    return (t.contiguous().view(torch.int32) & ~0x1FFF).view(torch.float32)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows", [1, 300, 4096])
def test_epilogue_is_the_unfused_residual_add_bit_for_bit(dtype, rows):
    n = 512
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = torch.randn(rows, n, device="cuda", generator=g)
    x = (_tf32_exact(x) if dtype == torch.float32 else x).to(dtype)
    eye = torch.eye(n, device="cuda", dtype=dtype)
    bias = torch.randn(n, device="cuda", generator=g).to(dtype)
    res = (3 * torch.randn(rows, n, device="cuda", generator=g)).to(dtype)
    out = fused_linear_residual(x, eye, bias, res)
    assert torch.equal(out, res + (x + bias))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize(
    "rows,k,n", [(256, 768, 768), (1000, 768, 768), (513, 3072, 768), (77, 72, 200), (2048, 256, 1024)]
)
def test_gemm_is_within_its_rounding_bound(dtype, rows, k, n):
    g = torch.Generator(device="cuda").manual_seed(rows + k + n)
    x = torch.randn(rows, k, device="cuda", generator=g).to(dtype)
    bound = k ** -0.5
    w = ((torch.rand(n, k, device="cuda", generator=g) * 2 - 1) * bound).to(dtype)
    b = ((torch.rand(n, device="cuda", generator=g) * 2 - 1) * bound).to(dtype)
    res = torch.randn(rows, n, device="cuda", generator=g).to(dtype)
    out = fused_linear_residual(x, w, b, res).double()
    xd, wd = x.double(), w.double()
    exact = res.double() + xd @ wd.T + b.double()
    mag = xd.abs() @ wd.abs().T
    u = UNIT[dtype]
    if dtype == torch.float32:
        # both operands truncated to TF32 (2^-10 relative each), fp32 sums
        tol = 2.5 * u * mag + 2.0 ** -22 * (res.double().abs() + mag + b.double().abs())
    else:
        # projection rounded to the format, sum rounded again, fp32 accumulation
        proj = xd @ wd.T + b.double()
        tol = u * proj.abs() + u * exact.abs() + 2.0 ** -20 * (mag + 1)
    assert bool(((out - exact).abs() <= tol + 1e-30).all())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_invalid_rows_are_zeroed_and_the_residual_may_be_the_output(dtype):
    rows, k, n = 600, 256, 768
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(rows, k, device="cuda", generator=g).to(dtype)
    w = (torch.randn(n, k, device="cuda", generator=g) / 16).to(dtype)
    b = torch.randn(n, device="cuda", generator=g).to(dtype)
    res = torch.randn(rows, n, device="cuda", generator=g).to(dtype)
    valid = torch.rand(rows, device="cuda", generator=g) > 0.3
    plain = fused_linear_residual(x, w, b, res)
    masked = fused_linear_residual(x, w, b, res, valid)
    assert torch.equal(masked[valid], plain[valid])
    assert torch.count_nonzero(masked[~valid]) == 0
    inplace = res.clone()
    assert fused_linear_residual(x, w, b, inplace, out=inplace) is inplace
    assert torch.equal(inplace, plain)


def test_unsupported_shapes_raise():
    x = torch.randn(4, 6, device="cuda")  # 24-byte rows
    with pytest.raises(ValueError, match="16 bytes"):
        fused_linear_residual(x, torch.randn(8, 6, device="cuda"), None, torch.randn(4, 8, device="cuda"))
    x = torch.randn(4, 8, device="cuda")
    with pytest.raises(ValueError, match="residual"):
        fused_linear_residual(x, torch.randn(8, 8, device="cuda"), None, torch.randn(4, 4, device="cuda"))
