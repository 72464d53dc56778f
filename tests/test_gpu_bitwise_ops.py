"""Every op of the fused bf16 forward other than attention reproduces the
explicit model's op bit for bit at the BASELINE model shapes (C3: d_model
4096, FFN 16384; C5: d_model 768, FFN 3072), so that the model-level
comparison with the explicit model isolates the attention kernel:

  * LayerNorm / residual + LayerNorm: statistics in the order of ATen's
    vectorised kernel (benchmarks/torch_transformer_benchmark.py:140-141 use
    nn.LayerNorm), equal to F.layer_norm bit for bit;
  * out_proj / ffn_out + residual (tcgen05 GEMM, residual epilogue) against
    ``res + F.linear(x, w, b)`` (cuBLAS), bit for bit at these shapes: both
    accumulate in fp32 over K in the same order;
  * the FFN input projection + GELU against ``F.gelu(F.linear(...))``: the
    GEMM is exact in the same sense; the 16-bit GELU is a polynomial erfc
    within one output unit of ATen's erf form and equal to it on nearly every
    element (differences that downstream sums absorb: the model-level op swap
    shows no change in the block outputs).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from transformer_opt.kernels import (
    fused_linear_gelu,
    fused_linear_residual,
    fused_residual_layer_norm,
    layer_norm,
)

pytestmark = pytest.mark.gpu

SHAPES = {"C5": (32768, 768, 3072), "C3": (16384, 4096, 16384)}  # rows, d_model, ffn


def _linear(n, k, g):
    bound = k ** -0.5  # nn.Linear's default init
    w = ((torch.rand(n, k, device="cuda", generator=g) * 2 - 1) * bound).to(torch.bfloat16)
    b = ((torch.rand(n, device="cuda", generator=g) * 2 - 1) * bound).to(torch.bfloat16)
    return w, b


@pytest.mark.parametrize("name", list(SHAPES))
def test_block_ops_equal_the_explicit_ops_bit_for_bit(name):
    rows, d, ffn = SHAPES[name]
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16)
    ln_w = torch.ones(d, device="cuda", dtype=torch.bfloat16)
    ln_b = torch.zeros(d, device="cuda", dtype=torch.bfloat16)
    w_o, b_o = _linear(d, d, g)
    w_in, b_in = _linear(ffn, d, g)
    w_out, b_out = _linear(d, ffn, g)
    with torch.inference_mode():
        h = layer_norm(x, ln_w, ln_b, 1e-5)
        assert torch.equal(h, F.layer_norm(x, (d,), ln_w, ln_b, 1e-5))
        ctx = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16) * 0.1
        x1 = fused_linear_residual(ctx, w_o, b_o, x)
        assert torch.equal(x1, x + F.linear(ctx, w_o, b_o))
        h2 = layer_norm(x1, ln_w, ln_b, 1e-5)
        assert torch.equal(h2, F.layer_norm(x1, (d,), ln_w, ln_b, 1e-5))
        r, n = fused_residual_layer_norm(x, F.linear(ctx, w_o, b_o), ln_w, ln_b, 1e-5)
        assert torch.equal(r, x1) and torch.equal(n, h2)
        hidden = fused_linear_gelu(h2, w_in, b_in)
        ref = F.gelu(F.linear(h2, w_in, b_in), approximate="none")
        differ = hidden != ref
        assert differ.float().mean().item() < 1e-4
        ulp = torch.finfo(torch.bfloat16).eps * ref.float().abs().clamp_min(2.0 ** -126)
        assert bool(((hidden.float() - ref.float()).abs()[differ] <= ulp[differ]).all())
        x2 = fused_linear_residual(hidden, w_out, b_out, x1)
        assert torch.equal(x2, x1 + F.linear(hidden, w_out, b_out))


@pytest.mark.parametrize("name", list(SHAPES))
def test_packed_qkv_projection_equals_the_three_projections(name):
    rows, d, _ = SHAPES[name]
    g = torch.Generator(device="cuda").manual_seed(d)
    h = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16)
    parts = [_linear(d, d, g) for _ in range(3)]
    packed = F.linear(h, torch.cat([w for w, _ in parts]), torch.cat([b for _, b in parts]))
    for i, (w, b) in enumerate(parts):
        assert torch.equal(packed[:, i * d:(i + 1) * d], F.linear(h, w, b))
