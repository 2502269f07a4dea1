"""Build oracle/_ref/libmetal_ref.so: the reference's Metal decode kernel body run on the CPU.

TEST INFRASTRUCTURE ONLY. Reads the kernel body string (_PAGED_DECODE_SOURCE)
from the reference checkout without importing it (mlx is not installed), writes
it to oracle/_ref/paged_decode_body.inc (git-ignored, never committed) and
compiles oracle/metal_ref/metal_shim.cpp around it with g++.

    python oracle/metal_ref/build.py --reference /path/to/mini-sglang-mlx
    MINISGL_REFERENCE=/path/to/mini-sglang-mlx python oracle/metal_ref/build.py

The checkout is named only by --reference or the MINISGL_REFERENCE
environment variable. Without one (e.g. on a GPU host that has no checkout)
the prebuilt library, if any, is used as is.
"""

from __future__ import annotations

import argparse
import ast
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = ROOT / "oracle" / "_ref"
LIB = OUT / "libmetal_ref.so"
KERNEL_FILE = Path("python/minisgl_mlx/attention/metal.py")


def extract_body(reference: Path) -> str:
    tree = ast.parse((reference / KERNEL_FILE).read_text())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", "") == "_PAGED_DECODE_SOURCE" for t in node.targets):
            return node.value.value
    raise RuntimeError(f"_PAGED_DECODE_SOURCE not found in {reference / KERNEL_FILE}")


def default_reference() -> Path | None:
    env = os.environ.get("MINISGL_REFERENCE")
    return Path(env) if env else None


def build(reference: Path | None = None, quiet: bool = False) -> Path | None:
    reference = reference or default_reference()
    if reference is None or not (reference / KERNEL_FILE).exists():
        return LIB if LIB.exists() else None
    OUT.mkdir(parents=True, exist_ok=True)
    body = extract_body(reference)
    inc = OUT / "paged_decode_body.inc"
    if not inc.exists() or inc.read_text() != body:
        inc.write_text(body)
    src = HERE / "metal_shim.cpp"
    if LIB.exists() and LIB.stat().st_mtime > max(src.stat().st_mtime, inc.stat().st_mtime):
        return LIB
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-I", str(OUT), "-o", str(LIB), str(src)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"metal_ref build failed:\n{res.stderr}")
    if not quiet:
        print(LIB, file=sys.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    args = ap.parse_args()
    print(build(args.reference))
