"""UserOptimizedTransformer on CPU against the oracle's explicit model
(the reference's tests/test_correctness.py strategy, :26-110)."""

from __future__ import annotations

import itertools

import pytest
import torch

from oracle import explicit as oracle
from tests import _golden
from transformer_opt.submission import TransformerConfig, UserOptimizedTransformer

SHAPES = [
    (1, 32, 64, 4, 256, 2),
    (8, 128, 256, 8, 1024, 2),
    (2, 96, 128, 8, 512, 3),
    (4, 64, 512, 8, 1024, 1),
]


def _pair(b, s, d, h, f, layers, causal, seed=0):
    torch.manual_seed(seed)
    baseline = oracle.BaselineTransformer(oracle.TransformerConfig(b, s, d, h, f, layers, causal)).eval()
    optimized = UserOptimizedTransformer(TransformerConfig(b, s, d, h, f, layers, causal)).eval()
    oracle.copy_model_weights(baseline, optimized, strict=True)
    return baseline, optimized


@pytest.mark.parametrize(
    "shape,causal,padding", list(itertools.product(SHAPES, [False, True], [0.0, 0.3])), ids=str
)
def test_cpu_forward_matches_oracle(shape, causal, padding):
    baseline, optimized = _pair(*shape, causal)
    cfg = oracle.TransformerConfig(*shape, causal)
    x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, 7, padding)
    with torch.inference_mode():
        ref = baseline(x, mask)
        opt = optimized(x, mask)
    res = oracle.compare_outputs(ref, opt)
    assert res.passed, res
    assert optimized.attention_backend_counts["reference"] == shape[-1]


def test_state_dict_is_interchangeable_both_ways():
    baseline, optimized = _pair(2, 16, 64, 8, 128, 2, False)
    assert list(baseline.state_dict()) == list(optimized.state_dict())
    baseline.load_state_dict(optimized.state_dict(), strict=True)


def test_same_seed_gives_same_initialisation():
    cfg = (2, 16, 64, 4, 128, 2, True)
    torch.manual_seed(123)
    baseline = oracle.BaselineTransformer(oracle.TransformerConfig(*cfg))
    torch.manual_seed(123)
    optimized = UserOptimizedTransformer(TransformerConfig(*cfg))
    for (n1, t1), (n2, t2) in zip(baseline.state_dict().items(), optimized.state_dict().items()):
        assert n1 == n2 and torch.equal(t1, t2)


def test_golden_model_case_through_optimized_model():
    data = _golden.load("model.npz")
    b, s, dm, h, f, layers, causal, seed = (int(v) for v in data["m1_cfg"])
    torch.manual_seed(seed)
    model = UserOptimizedTransformer(TransformerConfig(b, s, dm, h, f, layers, bool(causal))).eval()
    x = torch.from_numpy(data["m1_x"])
    mask = torch.from_numpy(data["m1_mask"])
    with torch.inference_mode():
        y = model(x, mask)
    res = oracle.compare_outputs(torch.from_numpy(data["m1_y"]), y)
    assert res.passed, res


def test_explicit_all_valid_mask_matches_none():
    _, optimized = _pair(2, 33, 64, 4, 128, 1, True)
    x = torch.randn(2, 33, 64)
    with torch.inference_mode():
        a = optimized(x, None)
        b = optimized(x, torch.ones(2, 33, dtype=torch.bool))
    assert oracle.compare_outputs(a, b).passed


def test_constructor_validation():
    cfg = TransformerConfig(1, 8, 16, 2, 32, 1, False)
    with pytest.raises(ValueError, match="attention_backend"):
        UserOptimizedTransformer(cfg, attention_backend="mystery")
    with pytest.raises(ValueError, match="execution_mode"):
        UserOptimizedTransformer(cfg, execution_mode="never")
    for mode in ("auto", "eager", "graph"):
        assert UserOptimizedTransformer(cfg, execution_mode=mode).execution_mode == mode
    with pytest.raises(ValueError, match="ffn_backend"):
        UserOptimizedTransformer(cfg, ffn_backend="cublaslt")
    for backend in ("auto", "b200", "torch"):
        model = UserOptimizedTransformer(cfg, ffn_backend=backend)
        assert model.ffn_backend == backend and model.fused_linear_gelu_calls == 0


def test_ffn_backend_is_keyword_only_and_cpu_forward_ignores_it():
    cfg = TransformerConfig(1, 8, 16, 2, 32, 1, False)
    with pytest.raises(TypeError):
        UserOptimizedTransformer(cfg, "auto", "auto", "torch")
    x = torch.randn(1, 8, 16)
    fused = UserOptimizedTransformer(cfg, ffn_backend="b200").eval()
    plain = UserOptimizedTransformer(cfg, ffn_backend="torch").eval()
    plain.load_state_dict(fused.state_dict(), strict=True)
    with torch.inference_mode():
        assert torch.equal(fused(x), plain(x))
    assert fused.fused_linear_gelu_calls == 0  # CPU: explicit forward, no kernel


def test_graph_mode_on_cpu_runs_the_explicit_forward():
    cfg = TransformerConfig(1, 8, 16, 2, 32, 1, False)
    model = UserOptimizedTransformer(cfg, execution_mode="graph").eval()
    with torch.inference_mode():
        out = model(torch.randn(1, 8, 16))
    assert out.shape == (1, 8, 16)
    assert model.cuda_graph_replays == 0


def test_fused_route_reason_on_cpu():
    model = UserOptimizedTransformer(TransformerConfig(1, 8, 16, 2, 32, 1, False)).eval()
    assert model.fused_route_reason(torch.randn(1, 8, 16), None) == "CPU input"
    sdpa = UserOptimizedTransformer(TransformerConfig(1, 8, 16, 2, 32, 1, False), "sdpa")
    assert "explicit math" in sdpa.fused_route_reason(torch.randn(1, 8, 16), None)


def test_forward_host_on_a_cpu_model_is_forward():
    cfg = TransformerConfig(4, 8, 16, 2, 32, 1, False)
    model = UserOptimizedTransformer(cfg).eval()
    x = torch.randn(4, 8, 16)
    with torch.inference_mode():
        ref = model(x)
        assert torch.equal(model.forward_host(x, chunks=2), ref)
        out = torch.empty_like(x)
        assert model.forward_host(x, out=out) is out and torch.equal(out, ref)


def test_default_host_chunks_keep_whole_sequences_and_enough_elements():
    chunks = UserOptimizedTransformer.default_host_chunks
    assert chunks(8, 2048) == 4      # 2 sequences (4096 tokens x 1024) per chunk
    assert chunks(512, 512) == 8     # capped at 8 chunks
    assert chunks(4, 16384) == 4     # one sequence per chunk
    assert chunks(4, 512) == 1       # too few elements to split at width 1024
    assert chunks(4, 512, 4096) == 2  # ... but enough at d_model 4096 (C4)
    assert chunks(7, 4096) == 7      # divisors of the batch only
    assert chunks(7, 2048) == 1
    assert chunks(1, 1) == 1
    plan = UserOptimizedTransformer.default_host_plan
    assert plan(8, 2048, 1024) == [1, 2, 2, 2, 1]          # C2: halves keep 2048 x 1024
    assert plan(512, 512, 768) == [32] + [64] * 7 + [32]   # C5
    assert plan(4, 16384, 4096) == [1, 1, 1, 1]            # C3: a sequence cannot be halved
    assert plan(4, 512, 4096) == [1, 2, 1]                 # C4
    assert plan(2, 128, 256) == [2]                        # C1: one chunk
    assert plan(8, 1024, 1024) == [2, 4, 2]                # 4-sequence chunks, halved ends
    assert sum(plan(512, 512, 768)) == 512


def test_forward_host_accepts_chunk_sizes_on_a_cpu_model():
    cfg = TransformerConfig(4, 8, 16, 2, 32, 1, False)
    model = UserOptimizedTransformer(cfg).to("cpu").eval()
    x = torch.randn(4, 8, 16)
    with torch.inference_mode():
        ref = model(x)
        assert torch.equal(model.forward_host(x, chunks=[1, 3]), ref)  # CPU: plain forward


def test_tf32_weight_rounding_keeps_nan_and_rounds_like_the_hardware():
    import struct

    from transformer_opt.submission import _round_to_tf32

    def rna_tf32(value: float) -> float:
        # round to 10 explicit mantissa bits, ties away from zero, on the bits
        (bits,) = struct.unpack("<I", struct.pack("<f", value))
        sign, mag = bits & 0x80000000, bits & 0x7FFFFFFF
        if mag > 0x7F800000:
            return value  # NaN stays NaN
        mag = min(((mag + 0x1000) & ~0x1FFF), 0x7F800000)
        return struct.unpack("<f", struct.pack("<I", sign | mag))[0]

    flt_max = torch.finfo(torch.float32).max
    values = torch.tensor(
        [1.0, -1.0, 1.0 + 2**-11, 1.0 + 3 * 2**-12, -(1.0 + 2**-11), flt_max, -flt_max,
         float("inf"), float("-inf"), 1e-40, -3.14159, 65504.0, 0.0, -0.0],
        dtype=torch.float32,
    )
    rounded = _round_to_tf32(values)
    for v, r in zip(values.tolist(), rounded.tolist()):
        assert r == rna_tf32(v) or (r != r and v != v), (v, r)
    assert torch.isinf(rounded[5]) and rounded[5] > 0  # FLT_MAX carries to +inf
    # NaN payloads whose integer carry would wrap into an infinity or a zero
    nan_bits = torch.tensor([0x7FFFF000, 0x7FFFFFFF, -4096, 0x7F801000], dtype=torch.int32)
    nans = nan_bits.view(torch.float32)
    assert torch.isnan(_round_to_tf32(nans)).all()


def test_check_device_status_is_a_no_op_off_cuda():
    model = UserOptimizedTransformer(TransformerConfig(1, 8, 16, 2, 32, 1, False))
    model.check_device_status()
    model.check_device_status(clear=True)
