"""Loading helpers for the golden vectors under tests/golden/."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def load(name: str):
    return np.load(GOLDEN / name, allow_pickle=False)


def tensor(arr: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype in (torch.float16, torch.bfloat16):
        return torch.from_numpy(arr.astype(np.uint16).view(np.int16).copy()).view(dtype)
    return torch.from_numpy(np.array(arr)).to(dtype)


def attention_cases():
    data = load("attention.npz")
    keys = sorted({k.split("_")[0] for k in data.files})
    cases = []
    for key in keys:
        b, s, h, d, causal = (int(v) for v in data[f"{key}_meta"])
        dtype = DTYPES[str(data[f"{key}_dtype"])]
        mask = torch.from_numpy(data[f"{key}_mask"]) if f"{key}_mask" in data.files else None
        cases.append(
            dict(
                key=key, shape=(b, s, h, d), causal=bool(causal), dtype=dtype,
                q=tensor(data[f"{key}_q"], dtype), k=tensor(data[f"{key}_k"], dtype),
                v=tensor(data[f"{key}_v"], dtype), out=tensor(data[f"{key}_out"], dtype),
                mask=mask,
            )
        )
    return cases


def rln_cases():
    data = load("rln.npz")
    keys = sorted({"_".join(k.split("_")[:2]) for k in data.files})
    cases = []
    for key in keys:
        dtype = DTYPES[key.split("_")[1]]
        masked, zr, zn = (bool(v) for v in data[f"{key}_flags"])
        case = dict(key=key, dtype=dtype, zero_residual=zr, zero_normalized=zn)
        for name in ("x", "u", "w", "b", "res", "norm"):
            case[name] = tensor(data[f"{key}_{name}"], dtype)
        case["mask"] = torch.from_numpy(data[f"{key}_mask"]) if masked else None
        cases.append(case)
    return cases


def assert_close_to_golden(actual: torch.Tensor, golden: torch.Tensor, what: str) -> None:
    """Golden outputs came from the reference's code on the host that ran
    make_golden.py. CPU GEMM kernels round differently across instruction sets
    (AVX2 / AVX-512 paths of the BLAS), so on another host the same code lands
    within a couple of units in the last place of the output's scale, not on
    the same bits. Bound: |actual - golden| <= 2 * eps(dtype) * max|golden|.
    The bitwise claim (oracle == reference on one host) is make_golden.py
    --check."""
    assert actual.dtype == golden.dtype and actual.shape == golden.shape, what
    a, g = actual.float(), golden.float()
    scale = float(g.abs().max()) if g.numel() else 0.0
    bound = 2.0 * torch.finfo(golden.dtype).eps * max(scale, 1e-30)
    err = float((a - g).abs().max()) if g.numel() else 0.0
    assert bool(torch.isfinite(a).eq(torch.isfinite(g)).all()), f"{what}: non-finite pattern differs"
    assert err <= bound, f"{what}: max |diff| {err:.3g} > {bound:.3g}"
