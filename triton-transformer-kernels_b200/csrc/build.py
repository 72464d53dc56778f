"""Build libb200tk.so (sm_100a) in-tree with nvcc.

Objects go to ``_build/`` beside this file; the shared library lands in
``../transformer_opt/kernels/libb200tk.so`` where the Python host package
loads it. The build is incremental on file modification times.

Usage: ``python build.py [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
REPO_ROOT = PKG_ROOT.parent
BUILD_DIR = CSRC / "_build"
OUTPUT = PKG_ROOT / "transformer_opt" / "kernels" / "libb200tk.so"
# (source, object stem, extra nvcc flags). attention_tc_inst.cu is compiled
# once per (dtype, head_dim) so the tcgen05 variants build in parallel.
UNITS = [
    ("capi.cu", "capi", ()),
    ("attention_tc.cu", "attention_tc", ()),
    ("attention_resident.cu", "attention_resident", ()),
    ("attention_generic.cu", "attention_generic", ()),
    ("residual_layer_norm.cu", "residual_layer_norm", ()),
    ("linear_gelu.cu", "linear_gelu", ()),
] + [
    (
        "attention_tc_inst.cu",
        f"attention_tc_{name}_d{hd}",
        (f"-DB200TK_TC_DTYPE={code}", f"-DB200TK_TC_HEAD_DIM={hd}"),
    )
    for code, name in ((0, "f32"), (1, "f16"), (2, "bf16"))
    for hd in (64, 128)
]
SOURCES = tuple(sorted({u[0] for u in UNITS}))
HEADERS = ("attention.h", "attention_tc.cuh", "attention_resident.cuh", "ptx_sm100.cuh")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
COMMON_FLAGS = (
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-diag-suppress",
    "177",
)


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _newest_input_mtime() -> float:
    files = [CSRC / s for s in SOURCES + HEADERS] + [REPO_ROOT / "include" / "b200tk.h"]
    return max(f.stat().st_mtime for f in files)


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> Path:
    """Compile every source for sm_100a and link the shared library."""
    if not force and OUTPUT.exists() and OUTPUT.stat().st_mtime >= _newest_input_mtime():
        return OUTPUT
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    header_mtime = max((CSRC / h).stat().st_mtime for h in HEADERS)

    def compile_one(unit) -> Path:
        src, stem, extra = unit
        obj = BUILD_DIR / (stem + ".o")
        if (
            not force
            and obj.exists()
            and obj.stat().st_mtime >= max((CSRC / src).stat().st_mtime, header_mtime)
        ):
            return obj
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{result.stdout}\n{result.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=max(1, jobs)) as pool:
        objects = list(pool.map(compile_one, UNITS))
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(tmp)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, OUTPUT)
    return OUTPUT


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
