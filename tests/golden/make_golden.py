"""Generate tests/golden/paged_decode_metal_ref.npz from the reference's own kernel.

Runs the reference's Metal paged-decode kernel body on the CPU
(oracle/metal_ref, built from python/minisgl_mlx/attention/metal.py of the
reference checkout) on the reference test's case list
(tests/test_attention.py:19-32: head shapes x {fp32, bf16}, B=7,
lens [1, 2, 17, 31, 32, 33, 700] on disjoint permuted slots). Inputs are drawn
from numpy default_rng(seed) and are NOT stored: the fixture keeps the
outputs plus a SHA-256 of every input array so a changed random stream is
detected. N is 2048 slots to keep the run short.

    python oracle/metal_ref/build.py && python tests/golden/make_golden.py
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import attention as O  # noqa: E402

SHAPES = [(16, 8, 128), (32, 8, 128), (8, 8, 64), (16, 2, 256)]
DTYPES = ["float32", "bfloat16"]
LENS = [1, 2, 17, 31, 32, 33, 700]
N = 2048
OUT = Path(__file__).resolve().parent / "paged_decode_metal_ref.npz"


def case_inputs(hq: int, hkv: int, d: int, dtype: str, seed: int):
    rng = np.random.default_rng(seed)
    k = O.round_to(rng.standard_normal((N, hkv, d)).astype(np.float32), dtype)
    v = O.round_to(rng.standard_normal((N, hkv, d)).astype(np.float32), dtype)
    q = O.round_to(rng.standard_normal((len(LENS), hq, d)).astype(np.float32), dtype)
    perm = rng.permutation(N).astype(np.int32)
    per, off = [], 0
    for n in LENS:
        per.append(perm[off:off + n])
        off += n
    indptr = np.concatenate([[0], np.cumsum(LENS)]).astype(np.int32)
    return q, k, v, indptr, np.concatenate(per).astype(np.int32), per


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def case_key(hq, hkv, d, dtype):
    return f"{hq}_{hkv}_{d}_{dtype}"


def main() -> None:
    from oracle.metal_ref import available, metal_paged_decode

    if not available():
        raise SystemExit("build oracle/_ref/libmetal_ref.so first (python oracle/metal_ref/build.py)")
    data = {}
    for i, (hq, hkv, d) in enumerate(SHAPES):
        for j, dt in enumerate(DTYPES):
            seed = 100 + 10 * i + j
            q, k, v, indptr, idx, _ = case_inputs(hq, hkv, d, dt, seed)
            out = metal_paged_decode(q, k, v, indptr, idx, d ** -0.5, dt)
            key = case_key(hq, hkv, d, dt)
            data[f"{key}_out"] = out.astype(np.float32)
            data[f"{key}_seed"] = np.array(seed)
            data[f"{key}_sha"] = np.array(digest(q, k, v, indptr, idx))
    np.savez_compressed(OUT, **data)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
