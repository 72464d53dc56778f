"""Fused residual + LayerNorm through libb200tk on a B200.

Mirrors the reference's tests/test_gpu_residual_layer_norm.py (:18-113):
the residual is exact (atol = rtol = 0), the normalized output within 1e-5
of F.layer_norm for fp32; 16-bit outputs within one rounding step of the
oracle (harness OR rule). Adds the golden vectors, 16-bit dtypes, the
BASELINE row widths at full row counts, ragged widths (scalar path) and the
plain-LayerNorm entry point.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import explicit as oracle
from tests import _golden
from transformer_opt.kernels import fused_residual_layer_norm, layer_norm

pytestmark = pytest.mark.gpu


def _contract(actual, reference):
    a, r = actual.float(), reference.float()
    err = (a - r).abs()
    ok = (err <= 1e-3) | (err <= 1e-2 * r.abs())
    assert ok.all(), f"failed={int((~ok).sum())} max_abs={err.max().item():.3g}"


@pytest.mark.parametrize("case", _golden.rln_cases(), ids=lambda c: c["key"])
def test_matches_reference_golden_vectors(case):
    x, u, w, b = (case[n].cuda() for n in ("x", "u", "w", "b"))
    mask = case["mask"].cuda() if case["mask"] is not None else None
    with torch.inference_mode():
        res, norm = fused_residual_layer_norm(
            x, u, w, b, 1e-5, mask,
            zero_invalid_residual=case["zero_residual"],
            zero_invalid_normalized=case["zero_normalized"],
        )
    assert torch.equal(res.cpu(), case["res"])
    if case["dtype"] == torch.float32:
        torch.testing.assert_close(norm.cpu(), case["norm"], rtol=1e-5, atol=1e-5)
    else:
        _contract(norm.cpu(), case["norm"])


@pytest.mark.parametrize(
    "masked,zero_residual,zero_normalized",
    [(False, False, False), (True, False, False), (True, True, False), (True, True, True)],
)
def test_matches_explicit_operations(masked, zero_residual, zero_normalized):
    torch.manual_seed(7018)
    x = torch.randn(2, 17, 128, device="cuda")
    u, w, b = torch.randn_like(x), torch.randn(128, device="cuda"), torch.randn(128, device="cuda")
    mask = None
    if masked:
        mask = torch.arange(17, device="cuda")[None, :] < torch.tensor([[17], [9]], device="cuda")
    exp_r, exp_n = oracle.residual_layer_norm(x, u, w, b, 1e-5, mask, zero_residual, zero_normalized)
    with torch.inference_mode():
        r, n = fused_residual_layer_norm(
            x, u, w, b, 1e-5, mask,
            zero_invalid_residual=zero_residual, zero_invalid_normalized=zero_normalized,
        )
    torch.testing.assert_close(r, exp_r, rtol=0, atol=0)
    torch.testing.assert_close(n, exp_n, rtol=1e-5, atol=1e-5)


def test_without_bias():
    torch.manual_seed(7019)
    x = torch.randn(3, 5, 128, device="cuda")
    u, w = torch.randn_like(x), torch.randn(128, device="cuda")
    with torch.inference_mode():
        r, n = fused_residual_layer_norm(x, u, w, None, 1e-5)
    torch.testing.assert_close(r, x + u, rtol=0, atol=0)
    torch.testing.assert_close(n, F.layer_norm(x + u, (128,), w, None, 1e-5), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("width", [8, 33, 100, 256, 768, 1000, 1024, 4096, 6144, 16384])
def test_widths_and_dtypes(width, dtype):
    torch.manual_seed(width)
    x = torch.randn(37, width, device="cuda", dtype=dtype)
    u = torch.randn_like(x)
    w = torch.randn(width, device="cuda", dtype=dtype)
    b = torch.randn(width, device="cuda", dtype=dtype)
    mask = torch.rand(37, device="cuda") > 0.3
    exp_r, exp_n = oracle.residual_layer_norm(x, u, w, b, 1e-5, mask, True, True)
    with torch.inference_mode():
        r, n = fused_residual_layer_norm(
            x, u, w, b, 1e-5, mask, zero_invalid_residual=True, zero_invalid_normalized=True
        )
    assert torch.equal(r, exp_r)
    if dtype == torch.float32:
        torch.testing.assert_close(n, exp_n, rtol=1e-5, atol=2e-5)
    else:
        _contract(n, exp_n)


def test_unaligned_views_take_the_scalar_path():
    torch.manual_seed(3)
    base = torch.randn(4 * 257 + 1, device="cuda")
    x = base[1:].view(4, 257)  # 4-byte offset: not 16-byte aligned
    u = torch.randn(4, 257, device="cuda")
    w, b = torch.randn(257, device="cuda"), torch.randn(257, device="cuda")
    with torch.inference_mode():
        r, n = fused_residual_layer_norm(x, u, w, b, 1e-5)
    exp_r, exp_n = oracle.residual_layer_norm(x, u, w, b, 1e-5)
    torch.testing.assert_close(r, exp_r, rtol=0, atol=0)
    torch.testing.assert_close(n, exp_n, rtol=1e-5, atol=2e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_plain_layer_norm(dtype):
    torch.manual_seed(11)
    x = torch.randn(64, 768, device="cuda", dtype=dtype)
    w = torch.randn(768, device="cuda", dtype=dtype)
    b = torch.randn(768, device="cuda", dtype=dtype)
    with torch.inference_mode():
        n = layer_norm(x, w, b, 1e-5)
    _contract(n, F.layer_norm(x, (768,), w, b, 1e-5))


@pytest.mark.parametrize(
    "rows,width,dtype",
    [(256, 256, torch.float32), (16384, 1024, torch.float32), (65536, 4096, torch.bfloat16),
     (2048, 4096, torch.float32), (262144, 768, torch.bfloat16)],
    ids=["C1", "C2", "C3", "C4", "C5"],
)
def test_baseline_config_rows_full_size(rows, width, dtype):
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = torch.randn(rows, width, device="cuda", dtype=dtype, generator=g)
    u = torch.randn(rows, width, device="cuda", dtype=dtype, generator=g)
    w = torch.ones(width, device="cuda", dtype=dtype)
    b = torch.zeros(width, device="cuda", dtype=dtype)
    with torch.inference_mode():
        r, n = fused_residual_layer_norm(x, u, w, b, 1e-5)
        exp_r, exp_n = oracle.residual_layer_norm(x, u, w, b, 1e-5)
    assert torch.equal(r, exp_r)
    _contract(n, exp_n)
    # size-independent properties of a LayerNorm with gamma=1, beta=0
    nf = n.float()
    assert nf.mean(dim=-1).abs().max().item() < 2e-2
    assert (nf.var(dim=-1, unbiased=False) - 1).abs().max().item() < 2e-2


def test_round_normalized_tf32_flag():
    """ROUND_TF32: normalized output = nearest TF32 value (ties away from
    zero) of the unrounded output; the residual is unchanged; fp32 only."""
    g = torch.Generator(device="cuda").manual_seed(21)
    for rows, width in ((300, 1024), (7, 1001)):  # vector path, scalar path
        x = torch.randn(rows, width, device="cuda", generator=g)
        u = torch.randn(rows, width, device="cuda", generator=g)
        w = torch.randn(width, device="cuda", generator=g)
        b = torch.randn(width, device="cuda", generator=g)
        r0, n0 = fused_residual_layer_norm(x, u, w, b, 1e-5)
        r1, n1 = fused_residual_layer_norm(x, u, w, b, 1e-5, round_normalized_tf32=True)
        expect = ((n0.view(torch.int32) + 0x1000) & -0x2000).view(torch.float32)
        assert torch.equal(r0, r1)
        assert torch.equal(n1, expect)
        assert not torch.equal(n0, n1)
    xb = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    wb = torch.ones(64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fused_residual_layer_norm(xb, xb, wb, None, 1e-5, round_normalized_tf32=True)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("width", [256, 768, 1024, 4096])
def test_layer_norm_equals_torch_bit_for_bit(dtype, width):
    # 16-bit rows of whole 4-element groups up to 4096 wide compute their
    # statistics in the order of ATen's LayerNorm: the plain LayerNorm and the
    # fused residual form (on the rounded residual) equal F.layer_norm exactly.
    g = torch.Generator(device="cuda").manual_seed(width)
    x = (torch.randn(4096, width, device="cuda", generator=g) * 1.7 + 0.3).to(dtype)
    u = torch.randn(4096, width, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(width, device="cuda", generator=g)).to(dtype)
    b = (0.1 * torch.randn(width, device="cuda", generator=g)).to(dtype)
    with torch.inference_mode():
        ref = F.layer_norm(x, (width,), w, b, 1e-5)
        assert torch.equal(layer_norm(x, w, b, 1e-5), ref)
        res, norm = fused_residual_layer_norm(x, u, w, b, 1e-5)
        assert torch.equal(res, x + u)
        assert torch.equal(norm, F.layer_norm(x + u, (width,), w, b, 1e-5))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_many_row_pairs_per_warp_bit_for_bit(dtype):
    # Many CTAs of row pairs (40001 rows: an odd last row), a ragged mask with
    # both zeroing flags, the plain LayerNorm and the fused form: all equal
    # torch's ops bit for bit.
    g = torch.Generator(device="cuda").manual_seed(40001)
    rows, width = 40001, 768
    x = torch.randn(rows, width, device="cuda", generator=g).to(dtype)
    u = torch.randn(rows, width, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(width, device="cuda", generator=g)).to(dtype)
    b = (0.1 * torch.randn(width, device="cuda", generator=g)).to(dtype)
    mask = torch.rand(rows, device="cuda", generator=g) > 0.2
    with torch.inference_mode():
        assert torch.equal(layer_norm(x, w, b, 1e-5), F.layer_norm(x, (width,), w, b, 1e-5))
        res, norm = fused_residual_layer_norm(x, u, w, b, 1e-5)
        assert torch.equal(res, x + u)
        assert torch.equal(norm, F.layer_norm(x + u, (width,), w, b, 1e-5))
        res, norm = fused_residual_layer_norm(x, u, w, b, 1e-5, mask,
                                              zero_invalid_residual=True,
                                              zero_invalid_normalized=True)
        keep = mask[:, None]
        expect_res = torch.where(keep, x + u, torch.zeros_like(x))
        assert torch.equal(res, expect_res)
        expect_norm = torch.where(keep, F.layer_norm(expect_res, (width,), w, b, 1e-5),
                                  torch.zeros_like(x))
        assert torch.equal(norm, expect_norm)
