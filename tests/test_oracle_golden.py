"""Pin the oracle to the reference: its outputs must reproduce the golden
vectors that tests/golden/make_golden.py produced by running the reference
project's own code (CPU, no GPU needed). Outputs that pass through a CPU GEMM
are held to a two-ulp bound of their scale (the BLAS rounds differently on
other instruction sets); the rest are compared bit for bit. Bitwise identity
of oracle and reference on one host is what ``make_golden.py --check``
verifies."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import explicit as oracle
from tests import _golden


@pytest.mark.parametrize("case", _golden.attention_cases(), ids=lambda c: c["key"])
def test_oracle_attention_matches_reference(case):
    with torch.inference_mode():
        out = oracle.reference_attention(
            case["q"], case["k"], case["v"], case["mask"], case["causal"], None
        )
    _golden.assert_close_to_golden(out, case["out"], f"attention {case['key']}")


@pytest.mark.parametrize("case", _golden.attention_cases()[:6], ids=lambda c: c["key"])
def test_oracle_row_subset_matches_full(case):
    s = case["shape"][1]
    rows = sorted({0, s // 3, s - 1})
    with torch.inference_mode():
        part = oracle.reference_attention_rows(
            case["q"], case["k"], case["v"], rows, case["mask"], case["causal"], None
        )
    torch.testing.assert_close(part.float(), case["out"][:, rows].float(), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("case", _golden.rln_cases(), ids=lambda c: c["key"])
def test_oracle_residual_layer_norm_matches_reference(case):
    res, norm = oracle.residual_layer_norm(
        case["x"], case["u"], case["w"], case["b"], 1e-5, case["mask"],
        case["zero_residual"], case["zero_normalized"],
    )
    assert torch.equal(res, case["res"])
    assert torch.equal(norm, case["norm"])


def _weights_digest(model) -> str:
    digest = hashlib.sha256()
    for name, t in model.state_dict().items():
        digest.update(name.encode())
        digest.update(t.numpy().tobytes())
    return digest.hexdigest()


@pytest.mark.parametrize("index", [0, 1, 2])
def test_oracle_model_matches_reference(index):
    data = _golden.load("model.npz")
    b, s, dm, h, f, layers, causal, seed = (int(v) for v in data[f"m{index}_cfg"])
    pad = float(data[f"m{index}_pad"])
    cfg = oracle.TransformerConfig(b, s, dm, h, f, layers, bool(causal))
    torch.manual_seed(seed)
    model = oracle.BaselineTransformer(cfg).eval()
    assert _weights_digest(model) == str(data[f"m{index}_weights_sha256"])
    x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed + 1, pad, 1.0)
    assert torch.equal(x, torch.from_numpy(data[f"m{index}_x"]))
    if pad > 0:
        assert torch.equal(mask, torch.from_numpy(data[f"m{index}_mask"]))
    else:
        assert mask is None
    with torch.inference_mode():
        y = model(x, mask)
    _golden.assert_close_to_golden(y, torch.from_numpy(data[f"m{index}_y"]), f"model {index}")


def test_oracle_compare_outputs_matches_reference():
    data = _golden.load("model.npz")
    ref, opt = torch.from_numpy(data["cmp_ref"]), torch.from_numpy(data["cmp_opt"])
    res = oracle.compare_outputs(ref, opt, rtol=0.01, atol=0.001)
    expected = data["cmp_result"]
    assert res.failed_elements == int(expected[0])
    assert res.total_elements == int(expected[1])
    assert res.max_abs_error == pytest.approx(expected[2], rel=1e-6)
    assert res.max_relative_error == pytest.approx(expected[3], rel=1e-6)
    assert res.mean_abs_error == pytest.approx(expected[4], rel=1e-6)
    assert res.worst_index == tuple(int(v) for v in expected[5:])
