"""Build the in-tree CUDA library ``minisgl_b200/libb200attn.so`` for sm_100a.

The library is a plain C-ABI shared object (include/b200attn.h) compiled by
nvcc in one translation unit. It is built in-tree so that it travels with the
source tree to the GPU host; nothing is installed into site-packages.

    python mini-sglang-mlx_b200/build.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_PATH = PKG_ROOT / "minisgl_b200" / "libb200attn.so"

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC,-O3",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > mtime for src in _sources())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not needs_build():
        return LIB_PATH
    cmd = [_nvcc(), *NVCC_FLAGS]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-I", str(INCLUDE), "-o", str(LIB_PATH) + ".tmp", str(CSRC / "b200attn.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_verbose:
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas))
