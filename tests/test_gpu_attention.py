"""Fused attention through libb200tk on a B200 against the oracle.

Mirrors the reference's tests/test_gpu_attention.py (cases :18-31, mask
modes :34-50, all-masked rows :114-128, causal tile frontier :153-169,
future-tile invariance :172-181) and adds the golden vectors produced by the
reference itself, packed-QKV strided views, the tcgen05 tile frontier, and
the BASELINE configurations at full size (checked on a subset of query rows,
which attention computes independently).

Tolerance: every element abs_err <= 1e-3 OR abs_err <= 1e-2 * |ref|
(the harness rule), outputs finite.
"""

from __future__ import annotations

import pytest
import torch

from oracle import explicit as oracle
from tests import _golden
from transformer_opt import attention_forward
from transformer_opt.kernels import _native, attention_route

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-2


@pytest.fixture(autouse=True, scope="module")
def _device_status_clean():
    _native.device_status(0, clear=True)
    yield
    assert _native.device_status(0) == 0, "a kernel recorded a pipeline timeout"


def assert_within_contract(actual: torch.Tensor, reference: torch.Tensor) -> None:
    a, r = actual.float(), reference.float()
    err = (a - r).abs()
    ok = (err <= ATOL) | (err <= RTOL * r.abs())
    assert torch.isfinite(a).all()
    assert ok.all(), f"failed={int((~ok).sum())}/{ok.numel()} max_abs={err.max().item():.3g}"


def run_b200(q, k, v, mask=None, causal=False, scale=None):
    with torch.inference_mode():
        out, decision = attention_forward(q, k, v, mask, causal=causal, scale=scale, backend="b200")
    assert decision.selected == "b200"
    return out


def make_mask(mode, batch, seq):
    if mode == "none":
        return None
    if mode == "all":
        return torch.ones(batch, seq, device="cuda", dtype=torch.bool)
    if mode == "minimum":
        lengths = torch.ones(batch, device="cuda", dtype=torch.long)
    else:
        lengths = torch.linspace(seq, max(1, seq // 2), batch, device="cuda").to(torch.long)
    return torch.arange(seq, device="cuda")[None, :] < lengths[:, None]


@pytest.mark.parametrize("case", _golden.attention_cases(), ids=lambda c: c["key"])
def test_matches_reference_golden_vectors(case):
    q, k, v = (case[n].cuda() for n in ("q", "k", "v"))
    mask = case["mask"].cuda() if case["mask"] is not None else None
    out = run_b200(q, k, v, mask, causal=case["causal"])
    assert out.dtype == case["out"].dtype
    assert_within_contract(out.cpu(), case["out"])


CASES = [
    (2, 31, 4, 8, torch.float16, True, "all", 1.0),
    (1, 65, 16, 8, torch.float32, True, "prefix", 1.0),
    (1, 1, 1, 16, torch.float16, False, "none", 1.0),
    (2, 31, 4, 32, torch.float16, True, "all", 1.0),
    (1, 63, 4, 64, torch.float16, False, "prefix", 0.25),
    (2, 64, 2, 64, torch.float16, True, "prefix", 1.0),
    (1, 65, 2, 128, torch.float16, False, "minimum", 1.0),
    (1, 127, 4, 32, torch.float16, True, "none", 3.0),
    (1, 129, 4, 64, torch.float16, True, "prefix", 1.0),
    (1, 257, 2, 32, torch.float16, False, "prefix", 1.0),
    (1, 65, 2, 32, torch.float32, True, "prefix", 1.0),
    # tcgen05 route: bf16 / fp16 / fp32 at head_dim 64 and 128
    (2, 300, 3, 64, torch.bfloat16, True, "prefix", 1.0),
    (2, 300, 3, 128, torch.bfloat16, False, "prefix", 1.0),
    (1, 513, 2, 64, torch.float32, True, "none", 1.0),
    (1, 513, 2, 128, torch.float32, False, "minimum", 1.0),
    (2, 257, 2, 128, torch.float16, True, "none", 1.0),
    (1, 1000, 2, 64, torch.float32, False, "prefix", 3.0),
]


@pytest.mark.parametrize("batch,seq,heads,dim,dtype,causal,mask_mode,scale_in", CASES)
def test_matches_explicit_reference(batch, seq, heads, dim, dtype, causal, mask_mode, scale_in):
    for seed in (7, 19):
        torch.manual_seed(seed)
        q = torch.randn(batch, seq, heads, dim, device="cuda", dtype=dtype) * scale_in
        k = torch.randn_like(q) * scale_in
        v = torch.randn_like(q)
        mask = make_mask(mask_mode, batch, seq)
        out = run_b200(q, k, v, mask, causal)
        with torch.inference_mode():
            ref = oracle.reference_attention(q, k, v, mask, causal)
        assert_within_contract(out, ref)


def test_all_keys_masked_rows_are_finite_zeros():
    for dim, dtype in ((32, torch.float16), (64, torch.bfloat16), (128, torch.float32)):
        q = torch.randn(2, 130, 2, dim, device="cuda", dtype=dtype)
        masked = torch.zeros(2, 130, device="cuda", dtype=torch.bool)
        out = run_b200(q, q, q, masked, causal=True)
        assert torch.isfinite(out).all()
        assert torch.count_nonzero(out) == 0


@pytest.mark.parametrize("seq", [1, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256, 257])
@pytest.mark.parametrize("dim", [32, 64, 128])
@pytest.mark.parametrize("mask_mode", ["none", "minimum"])
def test_causal_frontier_at_tile_boundaries(seq, dim, mask_mode):
    torch.manual_seed(41)
    q = torch.randn(1, seq, 2, dim, device="cuda")
    k, v = torch.randn_like(q), torch.randn_like(q)
    mask = make_mask(mask_mode, 1, seq)
    out = run_b200(q, k, v, mask, causal=True)
    with torch.inference_mode():
        ref = oracle.reference_attention(q, k, v, mask, True)
    assert_within_contract(out, ref)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dim,dtype", [(64, torch.float32), (128, torch.float32),
                                       (64, torch.bfloat16), (128, torch.float16)])
def test_padding_mask_only_changes_tiles_it_masks(dim, dtype, causal):
    # An all-valid mask takes the same arithmetic as no mask (bitwise), and
    # with a ragged mask the sequences whose keys are all valid match the
    # unmasked result bitwise too.
    torch.manual_seed(47)
    q = torch.randn(3, 300, 2, dim, device="cuda", dtype=dtype)
    k, v = torch.randn_like(q), torch.randn_like(q)
    plain = run_b200(q, k, v, causal=causal)
    all_valid = torch.ones(3, 300, device="cuda", dtype=torch.bool)
    assert torch.equal(run_b200(q, k, v, all_valid, causal=causal), plain)
    ragged = torch.arange(300, device="cuda")[None, :] < torch.tensor([[300], [171], [300]], device="cuda")
    out = run_b200(q, k, v, ragged, causal=causal)
    assert torch.equal(out[0], plain[0]) and torch.equal(out[2], plain[2])
    with torch.inference_mode():
        ref = oracle.reference_attention(q[1:2], k[1:2], v[1:2], ragged[1:2], causal)
    assert_within_contract(out[1:2], ref)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dim,dtype,seq,schedule", [
    (64, torch.float32, 700, "auto"), (128, torch.float32, 700, "auto"),
    (64, torch.bfloat16, 700, "two_pass"), (128, torch.bfloat16, 700, "one_pass"),
    (128, torch.float16, 700, "two_pass"), (64, torch.bfloat16, 500, "resident"),
    (64, torch.float16, 500, "resident"),
])
def test_key_tiles_wholly_past_the_padding_are_never_read(dim, dtype, seq, schedule, causal):
    # Right padding: key tiles that lie entirely past a row's last valid key
    # hold only zero probabilities, and the kernel neither loads nor
    # multiplies them. NaN in those tiles (positions from the 128-key
    # boundary after the last valid key on; every tile width divides 128)
    # therefore leaves the output bit-identical; the tile holding the boundary
    # is still read, so it gets large finite values that the mask zeroes.
    torch.manual_seed(59)
    batch = 5
    q = torch.randn(batch, seq, 2, dim, device="cuda", dtype=dtype)
    k, v = torch.randn_like(q), torch.randn_like(q)
    lengths = [seq, 131, 1, 0, 257]
    mask = torch.arange(seq, device="cuda")[None, :] < torch.tensor(lengths, device="cuda")[:, None]
    base = attention_fwd_with(q, k, v, mask, causal, schedule)
    for b, n in enumerate(lengths):
        k[b, n:] = 1e4
        v[b, n:] = -1e4
        end = -(-max(n, 1) // 128) * 128
        k[b, end:] = float("nan")
        v[b, end:] = float("nan")
    out = attention_fwd_with(q, k, v, mask, causal, schedule)
    assert torch.equal(out, base)
    assert torch.equal(out[3], torch.zeros_like(out[3]))  # no valid key: zeros
    if schedule == "one_pass":
        return  # its rounding meets the rule on long rows, not on these (see its own tests)
    with torch.inference_mode():
        ref = oracle.reference_attention(q[[0, 1, 2, 4]], k[[0, 1, 2, 4]].nan_to_num(),
                                         v[[0, 1, 2, 4]].nan_to_num(), mask[[0, 1, 2, 4]], causal)
    assert_within_contract(out[[0, 1, 2, 4]], ref)


@pytest.mark.parametrize("dtype,schedule", [(torch.bfloat16, "two_pass"), (torch.bfloat16, "resident"),
                                            (torch.float32, "auto")])
def test_masked_launch_beyond_the_per_batch_bound_table(dtype, schedule):
    # More batch rows than the kernels keep per-batch key bounds for (1024):
    # every key tile is computed, and the result is the same as on a batch
    # the table covers.
    torch.manual_seed(61)
    batch, seq = 1100, 200
    q = torch.randn(batch, seq, 1, 64, device="cuda", dtype=dtype)
    k, v = torch.randn_like(q), torch.randn_like(q)
    lengths = torch.randint(0, seq + 1, (batch,), device="cuda")
    mask = torch.arange(seq, device="cuda")[None, :] < lengths[:, None]
    out = attention_fwd_with(q, k, v, mask, False, schedule)
    rows = [0, 1, 517, 1023, 1024, 1099]
    part = attention_fwd_with(q[rows].contiguous(), k[rows].contiguous(), v[rows].contiguous(),
                              mask[rows].contiguous(), False, schedule)
    assert torch.equal(out[rows], part)
    valid = [r for r in rows if int(lengths[r]) > 0]
    with torch.inference_mode():
        ref = oracle.reference_attention(q[valid], k[valid], v[valid], mask[valid], False)
    assert_within_contract(out[valid], ref)


def attention_fwd_with(q, k, v, mask, causal, schedule):
    out = torch.empty_like(q)
    with torch.inference_mode():
        _native.attention_fwd(q, k, v, mask, out, causal, q.shape[-1] ** -0.5, schedule)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("scale", [0.3, -0.125])
@pytest.mark.parametrize("dim,dtype", [(64, torch.float32), (128, torch.float32), (64, torch.bfloat16)])
def test_custom_and_negative_scales(dim, dtype, scale):
    torch.manual_seed(53)
    q = torch.randn(2, 200, 2, dim, device="cuda", dtype=dtype)
    k, v = torch.randn_like(q), torch.randn_like(q)
    for causal in (False, True):
        out = run_b200(q, k, v, causal=causal, scale=scale)
        with torch.inference_mode():
            ref = oracle.reference_attention(q, k, v, None, causal, scale=scale)
        assert_within_contract(out, ref)


@pytest.mark.parametrize("dim,dtype", [(32, torch.float32), (64, torch.float32), (128, torch.bfloat16)])
def test_causal_future_tiles_are_never_observed(dim, dtype):
    torch.manual_seed(43)
    q = torch.randn(1, 300, 2, dim, device="cuda", dtype=dtype)
    k, v = torch.randn_like(q), torch.randn_like(q)
    before = run_b200(q, k, v, causal=True)
    k[:, 128:] *= 100
    v[:, 128:] += 100
    after = run_b200(q, k, v, causal=True)
    assert torch.equal(before[:, :128], after[:, :128])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [64, 128])
def test_packed_qkv_views_take_the_tcgen05_route(dtype, dim):
    torch.manual_seed(5)
    b, s, h = 2, 200, 3
    packed = torch.randn(b, s, 3, h, dim, device="cuda", dtype=dtype)
    q, k, v = packed.unbind(dim=2)
    assert attention_route(q, k, v) == "tcgen05"
    out = run_b200(q, k, v, causal=True)
    with torch.inference_mode():
        ref = oracle.reference_attention(q, k, v, None, True)
    assert_within_contract(out, ref)


def test_routes():
    q = torch.randn(1, 16, 2, 64, device="cuda", dtype=torch.bfloat16)
    assert attention_route(q, q, q) == "tcgen05"
    q32 = torch.randn(1, 16, 2, 32, device="cuda", dtype=torch.bfloat16)
    assert attention_route(q32, q32, q32) == "generic"
    big = torch.randn(1, 16, 2, 65, device="cuda", dtype=torch.bfloat16)[..., :64]
    assert attention_route(big, big, big) == "generic"  # 130-byte head stride: no TMA


def test_fp32_result_ignores_the_tf32_toggle():
    torch.manual_seed(29)
    q = torch.randn(1, 257, 2, 64, device="cuda")
    k, v = torch.randn_like(q), torch.randn_like(q)
    previous = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        a = run_b200(q, k, v, causal=True)
        torch.backends.cuda.matmul.allow_tf32 = True
        b = run_b200(q, k, v, causal=True)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous
    assert torch.equal(a, b)
    with torch.inference_mode():
        ref = oracle.reference_attention(q.double(), k.double(), v.double(), None, True)
    # 3xTF32 keeps fp32-level accuracy (TF32 alone would be ~1e-3 relative)
    assert (a.double() - ref).abs().max().item() < 2e-5


# BASELINE configurations (attention shapes per layer), full size.
FULL = {
    "C1": (2, 128, 4, 64, torch.float32, False),
    "C2": (8, 2048, 16, 64, torch.float32, True),
    "C3": (4, 16384, 32, 128, torch.bfloat16, True),
    "C4": (4, 512, 32, 128, torch.float32, False),
    "C5": (512, 512, 12, 64, torch.bfloat16, False),
}


@pytest.mark.parametrize("name", list(FULL))
def test_baseline_config_shapes_full_size(name):
    b, s, h, d, dtype, causal = FULL[name]
    g = torch.Generator(device="cuda").manual_seed(2024)
    scale_in = d**-0.5 if name == "C3" else 1.0
    q = (torch.randn(b, s, h, d, device="cuda", generator=g) * scale_in).to(dtype)
    k = (torch.randn(b, s, h, d, device="cuda", generator=g) * scale_in).to(dtype)
    v = (torch.randn(b, s, h, d, device="cuda", generator=g) * scale_in).to(dtype)
    out = run_b200(q, k, v, causal=causal)
    again = run_b200(q, k, v, causal=causal)
    assert torch.equal(out, again), "kernel is not deterministic"
    rows = sorted({0, 1, 127, 128, s // 2, s - 129, s - 128, s - 1} & set(range(s)))
    bsel = [0, b - 1] if b > 1 else [0]
    with torch.inference_mode():
        ref = oracle.reference_attention_rows(q[bsel], k[bsel], v[bsel], rows, None, causal)
    assert_within_contract(out[bsel][:, rows], ref)
    assert torch.isfinite(out).all()


def test_schedule_routing_by_sequence_length():
    # "auto": two passes (normalised probabilities rounded to the dtype, the
    # explicit math's rounding) below 4096 keys, one online pass from 4096 on
    from transformer_opt.kernels.attention import b200_attention

    torch.manual_seed(61)
    for seq, expected in ((1000, "two_pass"), (4096, "one_pass")):
        q = (torch.randn(1, seq, 2, 128, device="cuda") * 128 ** -0.5).to(torch.bfloat16)
        k, v = torch.randn_like(q), torch.randn_like(q)
        with torch.inference_mode():
            auto = b200_attention(q, k, v, causal=True)
            forced = b200_attention(q, k, v, causal=True, schedule=expected)
        assert torch.equal(auto, forced)
    q32 = torch.randn(1, 4096, 2, 64, device="cuda")  # fp32: one schedule only
    with torch.inference_mode():
        assert torch.equal(b200_attention(q32, q32, q32, schedule="one_pass"),
                           b200_attention(q32, q32, q32, schedule="two_pass"))


def test_c3_attention_meets_the_rule_on_every_element_five_seeds():
    # C3's attention (bf16, causal, S=16384, 32 heads, head_dim 128; q, k, v
    # ~ N(0,1) / sqrt(128)) on the schedule "auto" picks there (one pass),
    # every query row of every batch element against the explicit math.
    b, s, h, d = FULL["C3"][:4]
    for seed in range(5):
        g = torch.Generator(device="cuda").manual_seed(100 + seed)
        q, k, v = ((torch.randn(b, s, h, d, device="cuda", generator=g) * d ** -0.5)
                   .to(torch.bfloat16) for _ in range(3))
        out = run_b200(q, k, v, causal=True)
        for i in range(b):
            with torch.inference_mode():
                ref = oracle.reference_attention(q[i:i + 1], k[i:i + 1], v[i:i + 1], None, True)
            assert_within_contract(out[i:i + 1], ref)
            del ref
            torch.cuda.empty_cache()
