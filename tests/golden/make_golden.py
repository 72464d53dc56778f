"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference project's own code (imported from a checkout given with
``--reference``) on small seeded inputs and stores inputs and outputs under
this directory:

  attention.npz  : transformer_opt.dispatch._reference_attention on the
                   direct-kernel cases of tests/test_gpu_attention.py
                   (:18-31, mask modes :34-50) and its causal tile-frontier
                   sweep (:153-169), in float32 / float16 / bfloat16.
  rln.npz        : x + update and F.layer_norm with the masking variants of
                   tests/test_gpu_residual_layer_norm.py:18-81.
  model.npz      : benchmarks/torch_transformer_benchmark.py BaselineTransformer
                   (weights from torch.manual_seed) on generate_random_case
                   inputs, plus compare_outputs on a crafted pair.

16-bit tensors are stored as their raw uint16 bit patterns.
Usage: python tests/golden/make_golden.py --reference <reference checkout>
       [--check]

--check writes nothing: it runs the reference and the oracle (oracle/) on the
stored inputs on this host and requires their outputs to be bit-identical
(the golden files themselves may differ from both by the host's CPU GEMM
rounding when they were made on another instruction set).
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}

# (B, S, H, D, dtype, causal, mask mode, input scale)
ATTENTION_CASES = [
    (2, 31, 4, 8, "float16", True, "all", 1.0),
    (1, 65, 16, 8, "float32", True, "prefix", 1.0),
    (1, 1, 1, 16, "float16", False, "none", 1.0),
    (2, 31, 4, 32, "float16", True, "all", 1.0),
    (1, 63, 4, 64, "float16", False, "prefix", 0.25),
    (2, 64, 2, 64, "float16", True, "prefix", 1.0),
    (1, 65, 2, 128, "float16", False, "minimum", 1.0),
    (1, 127, 4, 32, "float16", True, "none", 3.0),
    (1, 129, 4, 64, "float16", True, "prefix", 1.0),
    (1, 257, 2, 32, "float16", False, "prefix", 1.0),
    (1, 65, 2, 32, "float32", True, "prefix", 1.0),
    # bfloat16 and the BASELINE head dims
    (2, 130, 2, 64, "bfloat16", True, "prefix", 1.0),
    (1, 200, 2, 128, "bfloat16", False, "none", 1.0),
    (1, 150, 2, 64, "float32", False, "minimum", 1.0),
    (1, 131, 2, 128, "float32", True, "none", 1.0),
] + [
    (1, s, 1, d, "float32", True, m, 1.0)
    for s in (31, 65, 129)
    for d in (32, 128)
    for m in ("none", "minimum")
]

MODEL_CASES = [
    # (B, S, d_model, H, ffn, layers, causal, padding_ratio, seed)
    (2, 128, 256, 4, 1024, 1, False, 0.0, 0),
    (2, 33, 64, 4, 128, 2, True, 0.3, 7),
    (1, 40, 64, 8, 96, 1, False, 0.25, 11),
]


def to_numpy(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def make_mask(mode: str, batch: int, seq: int):
    if mode == "none":
        return None
    if mode == "all":
        return torch.ones(batch, seq, dtype=torch.bool)
    if mode == "minimum":
        lengths = torch.ones(batch, dtype=torch.long)
    else:
        lengths = torch.linspace(seq, max(1, seq // 2), batch).to(torch.long)
    return torch.arange(seq)[None, :] < lengths[:, None]


def load_reference(root: Path):
    sys.path.insert(0, str(root))
    spec = importlib.util.spec_from_file_location(
        "benchmarks.torch_transformer_benchmark", root / "benchmarks" / "torch_transformer_benchmark.py"
    )
    organizer = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = organizer
    spec.loader.exec_module(organizer)
    from transformer_opt.dispatch import _reference_attention  # the reference's package

    return organizer, _reference_attention


def check(organizer, ref_attention) -> int:
    """Reference vs oracle, bit for bit, on the stored inputs (same host)."""
    sys.path.insert(0, str(HERE.parent.parent))
    sys.path.insert(0, str(HERE.parent))
    from oracle import explicit as oracle
    import _golden

    bad = 0
    for case in _golden.attention_cases():
        with torch.inference_mode():
            args = (case["q"], case["k"], case["v"], case["mask"], case["causal"], None)
            same = torch.equal(ref_attention(*args), oracle.reference_attention(*args))
        bad += not same
        print(f"attention {case['key']}: {'identical' if same else 'DIFFERENT'}")
    data = _golden.load("model.npz")
    for i, (b, s, dm, h, f, layers, causal, pad, seed) in enumerate(MODEL_CASES):
        outs = []
        for mod in (organizer, oracle):
            torch.manual_seed(seed)
            model = mod.BaselineTransformer(mod.TransformerConfig(b, s, dm, h, f, layers, causal)).eval()
            x = torch.from_numpy(data[f"m{i}_x"])
            mask = torch.from_numpy(data[f"m{i}_mask"]) if pad > 0 else None
            with torch.inference_mode():
                outs.append(model(x, mask))
        same = torch.equal(outs[0], outs[1])
        bad += not same
        print(f"model m{i}: {'identical' if same else 'DIFFERENT'}")
    print("all identical" if not bad else f"{bad} cases differ")
    return 1 if bad else 0


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True)
    parser.add_argument("--check", action="store_true")
    args = parser.parse_args()
    organizer, ref_attention = load_reference(args.reference.resolve())
    if args.check:
        return check(organizer, ref_attention)

    out = {}
    for i, (b, s, h, d, dt, causal, mode, scale_in) in enumerate(ATTENTION_CASES):
        g = torch.Generator().manual_seed(1000 + i)
        dtype = DTYPES[dt]
        q = (torch.randn(b, s, h, d, generator=g) * scale_in).to(dtype)
        k = (torch.randn(b, s, h, d, generator=g) * scale_in).to(dtype)
        v = torch.randn(b, s, h, d, generator=g).to(dtype)
        mask = make_mask(mode, b, s)
        with torch.inference_mode():
            o = ref_attention(q, k, v, mask, causal, None)
        key = f"a{i:02d}"
        out[f"{key}_meta"] = np.array([b, s, h, d, int(causal)], dtype=np.int64)
        out[f"{key}_dtype"] = np.array(dt)
        out[f"{key}_q"], out[f"{key}_k"], out[f"{key}_v"] = to_numpy(q), to_numpy(k), to_numpy(v)
        out[f"{key}_out"] = to_numpy(o)
        if mask is not None:
            out[f"{key}_mask"] = mask.numpy()
    np.savez_compressed(HERE / "attention.npz", **out)

    out = {}
    variants = [(False, False, False), (True, False, False), (True, True, False), (True, True, True)]
    for i, (masked, zr, zn) in enumerate(variants):
        for dt in ("float32", "bfloat16"):
            g = torch.Generator().manual_seed(7018 + i)
            dtype = DTYPES[dt]
            x = torch.randn(2, 17, 128, generator=g).to(dtype)
            u = torch.randn(2, 17, 128, generator=g).to(dtype)
            w = torch.randn(128, generator=g).to(dtype)
            bias = torch.randn(128, generator=g).to(dtype)
            mask = torch.arange(17)[None, :] < torch.tensor([[17], [9]]) if masked else None
            r = x + u
            if zr:
                r = r.masked_fill(~mask[..., None], 0)
            n = F.layer_norm(r, (128,), w, bias, 1e-5)
            if zn:
                n = n.masked_fill(~mask[..., None], 0)
            key = f"r{i}_{dt}"
            out[f"{key}_flags"] = np.array([int(masked), int(zr), int(zn)], dtype=np.int64)
            for name, t in (("x", x), ("u", u), ("w", w), ("b", bias), ("res", r), ("norm", n)):
                out[f"{key}_{name}"] = to_numpy(t)
            if mask is not None:
                out[f"{key}_mask"] = mask.numpy()
    np.savez_compressed(HERE / "rln.npz", **out)

    out = {}
    for i, (b, s, dm, h, f, layers, causal, pad, seed) in enumerate(MODEL_CASES):
        cfg = organizer.TransformerConfig(b, s, dm, h, f, layers, causal)
        torch.manual_seed(seed)
        model = organizer.BaselineTransformer(cfg).eval()
        digest = hashlib.sha256()
        for name, t in model.state_dict().items():
            digest.update(name.encode())
            digest.update(t.numpy().tobytes())
        x, mask = organizer.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed + 1, pad, 1.0)
        with torch.inference_mode():
            y = model(x, mask if pad > 0 else None)
        key = f"m{i}"
        out[f"{key}_cfg"] = np.array([b, s, dm, h, f, layers, int(causal), seed], dtype=np.int64)
        out[f"{key}_pad"] = np.array(pad)
        out[f"{key}_weights_sha256"] = np.array(digest.hexdigest())
        out[f"{key}_x"] = x.numpy()
        out[f"{key}_mask"] = mask.numpy()
        out[f"{key}_y"] = y.numpy()
    g = torch.Generator().manual_seed(5)
    ref = torch.randn(4, 6, 8, generator=g)
    opt = ref + torch.randn(4, 6, 8, generator=g) * 2e-3
    res = organizer.compare_outputs(ref, opt, rtol=0.01, atol=0.001)
    out["cmp_ref"], out["cmp_opt"] = ref.numpy(), opt.numpy()
    out["cmp_result"] = np.array(
        [res.failed_elements, res.total_elements, res.max_abs_error, res.max_relative_error,
         res.mean_abs_error] + list(res.worst_index), dtype=np.float64
    )
    np.savez_compressed(HERE / "model.npz", **out)
    for name in ("attention.npz", "rln.npz", "model.npz"):
        print(name, (HERE / name).stat().st_size, "bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
