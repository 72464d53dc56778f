"""Dispatch contract (CPU): mirrors the reference's tests/test_dispatch.py
portable cases (:18-47) for this package's backend names."""

from __future__ import annotations

import pytest
import torch

from transformer_opt import ATTENTION_BACKENDS, attention_forward, b200_attention_support
from transformer_opt import triton_attention_support
from transformer_opt.kernels import b200_attention


def _cpu_qkv(dtype=torch.float32):
    q = torch.randn(1, 8, 2, 16, dtype=dtype)
    return q, torch.randn_like(q), torch.randn_like(q)


def test_backend_names_are_a_superset_of_the_reference():
    assert {"auto", "triton", "sdpa", "reference"} <= set(ATTENTION_BACKENDS)
    assert "b200" in ATTENTION_BACKENDS


def test_cpu_auto_runs_explicit_reference_math():
    q, k, v = _cpu_qkv()
    output, decision = attention_forward(q, k, v, backend="auto")
    assert output.shape == q.shape
    assert decision.selected == "reference"
    assert "CUDA" in decision.reason


@pytest.mark.parametrize("backend", ["b200", "triton"])
def test_forced_custom_backend_fails_clearly_on_cpu(backend):
    q, k, v = _cpu_qkv()
    with pytest.raises(RuntimeError, match="custom attention was forced"):
        attention_forward(q, k, v, backend=backend)


def test_strict_kernel_wrapper_rejects_cpu_tensors():
    q, k, v = _cpu_qkv()
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        b200_attention(q, k, v)


def test_invalid_backend_is_rejected():
    q, k, v = _cpu_qkv()
    with pytest.raises(ValueError, match="attention backend"):
        attention_forward(q, k, v, backend="mystery")


def test_support_check_explains_bad_mask_shape():
    q, k, v = _cpu_qkv()
    result = b200_attention_support(q, k, v, torch.ones(1, 7, dtype=torch.bool))
    assert not result.supported
    assert "shape [batch, sequence]" in result.reason
    assert triton_attention_support is b200_attention_support


@pytest.mark.parametrize(
    "mutate,reason",
    [
        (lambda q, k, v: (q[..., :8], k, v), "identical shapes"),
        (lambda q, k, v: (q, k.double(), v), "identical dtypes"),
        (lambda q, k, v: (q.transpose(2, 3), k.transpose(2, 3), v.transpose(2, 3)), "stride must be 1"),
        (lambda q, k, v: (q[0], k[0], v[0]), "shape [batch, sequence, heads, head_dim]"),
    ],
)
def test_support_check_reports_contract_violations(mutate, reason):
    q, k, v = mutate(*_cpu_qkv())
    result = b200_attention_support(q, k, v)
    assert not result.supported
    assert reason in result.reason


def test_reference_and_sdpa_backends_agree_on_cpu():
    torch.manual_seed(3)
    q, k, v = _cpu_qkv()
    mask = torch.tensor([[True] * 6 + [False] * 2])
    ref, d1 = attention_forward(q, k, v, mask, causal=True, backend="reference")
    sdpa, d2 = attention_forward(q, k, v, mask, causal=True, backend="sdpa")
    assert (d1.selected, d2.selected) == ("reference", "sdpa")
    torch.testing.assert_close(ref, sdpa, rtol=1e-5, atol=1e-5)
