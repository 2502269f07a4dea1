"""Build (sm_100a) and run the tensor-core and exponential rate microbenchmarks.

These measure what bounds the extend kernel's 128-key block: tcgen05.mma at
the operand shapes it uses (and what a wait between MMA groups costs the
tensor pipe), 2^x on the MUFU and FMA pipes, and the latency of an mbarrier
wait.
Needs a B200; building alone (``--build-only``) needs only nvcc.
"""

from __future__ import annotations

import argparse
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE.parent / "csrc"
INCLUDE = HERE.parent.parent / "include"
BUILD = HERE / "_build"
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "--expt-relaxed-constexpr"]


def build() -> list[Path]:
    BUILD.mkdir(exist_ok=True)
    out = []
    for src in ("mma_rate.cu", "exp2_rate.cu", "mbar_wait_latency.cu"):
        exe = BUILD / src.replace(".cu", "")
        subprocess.run(["nvcc", *FLAGS, "-I", str(CSRC), "-I", str(INCLUDE), "-o", str(exe), str(HERE / src)],
                       check=True)
        out.append(exe)
    return out


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--build-only", action="store_true")
    args = ap.parse_args()
    exes = build()
    if args.build_only:
        return 0
    rc = 0
    for exe in exes:
        print(f"== {exe.name}", flush=True)
        rc |= subprocess.run([str(exe)]).returncode
    return rc


if __name__ == "__main__":
    sys.exit(main())
