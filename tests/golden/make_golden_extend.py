"""Generate tests/golden/extend_metal_ref.npz: ragged causal extend pinned to the reference's kernel.

The reference's prefill (python/minisgl_mlx/attention/base.py:85-105) runs one
causal SDPA per request: query row i of request r, whose prefix holds P_r
cached tokens, attends keys [0, P_r + i] (bottom-right alignment). Each such
row is exactly one decode over those P_r + i + 1 keys, and the reference's own
code computes that decode: its Metal paged-decode kernel body
(python/minisgl_mlx/attention/metal.py:35-95), executed on the CPU by
oracle/metal_ref. This script runs that kernel once per sampled query row, so
multi-token causal extend has vectors made by the reference's code rather than
by a restatement.

Batch: 10 requests with extend lengths 1, 2, 17, 127, 128, 129, 300, 64, 33, 5
(one-token, tile-boundary and long cases) over prefixes 0, 5, 33, 100, 16, 250,
3, 48, 0, 1000 (unaligned and page-aligned, with and without a prefix). The
token -> slot table hands each request whole 16-slot pages from a seeded
permutation of a 4096-slot pool, so the same table serves page sizes 16 and 1.
Cases: Hq/Hkv in {16/8, 32/8}, D = 128, float32 and bfloat16.

To keep the fixture small only some rows are stored: the first and last two of
each request, rows on either side of every 32-token boundary, and every 9th row;
each stored row carries all G query heads of one kv head (kv head = row % Hkv,
so every head is covered). The kernel is run per kv head on that head's slice of
the pools ([N, 1, D]), which is the arithmetic it performs for that head in a
full launch. Inputs are drawn from numpy default_rng(seed) and are NOT stored:
the fixture holds the outputs plus a SHA-256 of every input array.

    python oracle/metal_ref/build.py --reference <mini-sglang-mlx checkout>
    python tests/golden/make_golden_extend.py
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import attention as O  # noqa: E402

EXTEND = [1, 2, 17, 127, 128, 129, 300, 64, 33, 5]
PREFIX = [0, 5, 33, 100, 16, 250, 3, 48, 0, 1000]
SHAPES = [(16, 8, 128), (32, 8, 128)]
DTYPES = ["float32", "bfloat16"]
N = 4096
PAGE = 16
OUT = Path(__file__).resolve().parent / "extend_metal_ref.npz"


def sampled_rows(E: int) -> np.ndarray:
    i = np.arange(E)
    keep = (i < 2) | (i >= E - 2) | (i % 32 == 0) | (i % 32 == 31) | (i % 9 == 4)
    return i[keep]


def case_inputs(hq: int, hkv: int, d: int, dtype: str, seed: int):
    """Seeded q [T, Hq, D], pools [N, Hkv, D] and the token-granular table [B, max_len]."""
    rng = np.random.default_rng(seed)
    k = O.round_to(rng.standard_normal((N, hkv, d)).astype(np.float32), dtype)
    v = O.round_to(rng.standard_normal((N, hkv, d)).astype(np.float32), dtype)
    T = int(sum(EXTEND))
    q = O.round_to(rng.standard_normal((T, hq, d)).astype(np.float32), dtype)
    lens = np.array(PREFIX) + np.array(EXTEND)
    need = (lens + PAGE - 1) // PAGE
    free = rng.permutation(N // PAGE)
    table = np.zeros((len(lens), int(need.max()) * PAGE), np.int32)
    off = 0
    for b, n in enumerate(need.tolist()):
        table[b, : n * PAGE] = (free[off:off + n, None] * PAGE + np.arange(PAGE)[None, :]).reshape(-1)
        off += n
    return q, k, v, table


def sample_index(hkv: int):
    """(token index t in the packed batch, request, row i in the request, kv head) of every stored row."""
    rows = []
    t0 = 0
    for r, E in enumerate(EXTEND):
        for i in sampled_rows(E).tolist():
            rows.append((t0 + i, r, i, (t0 + i) % hkv))
        t0 += E
    return np.array(rows, dtype=np.int64)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def case_key(hq, hkv, d, dtype):
    return f"{hq}_{hkv}_{d}_{dtype}"


def run_reference_rows(q, k, v, table, hq, hkv, d, dtype, rows):
    """The reference kernel once per stored row: out [n_rows, G, D] (float32 carrier)."""
    from oracle.metal_ref import metal_paged_decode

    G = hq // hkv
    out = np.zeros((len(rows), G, d), np.float32)
    for h in range(hkv):
        sel = np.nonzero(rows[:, 3] == h)[0]
        if sel.size == 0:
            continue
        qh = np.ascontiguousarray(q[rows[sel, 0], h * G:(h + 1) * G, :])
        kh = np.ascontiguousarray(k[:, h:h + 1, :])
        vh = np.ascontiguousarray(v[:, h:h + 1, :])
        lens = np.array([PREFIX[r] + i + 1 for r, i in zip(rows[sel, 1], rows[sel, 2])], np.int64)
        indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        idx = np.concatenate([table[r, :n] for r, n in zip(rows[sel, 1], lens)]).astype(np.int32)
        out[sel] = metal_paged_decode(qh, kh, vh, indptr, idx, d ** -0.5, dtype)
    return out


def main() -> None:
    from oracle.metal_ref import available

    if not available():
        raise SystemExit("build oracle/_ref/libmetal_ref.so first (python oracle/metal_ref/build.py --reference ...)")
    data = {}
    for i, (hq, hkv, d) in enumerate(SHAPES):
        for j, dt in enumerate(DTYPES):
            seed = 500 + 10 * i + j
            q, k, v, table = case_inputs(hq, hkv, d, dt, seed)
            rows = sample_index(hkv)
            out = run_reference_rows(q, k, v, table, hq, hkv, d, dt, rows)
            key = case_key(hq, hkv, d, dt)
            if dt == "bfloat16":  # exact: the kernel rounds its output to bf16
                data[f"{key}_out_bf16bits"] = (out.view(np.uint32) >> 16).astype(np.uint16)
            else:
                data[f"{key}_out"] = out
            data[f"{key}_rows"] = rows.astype(np.int32)
            data[f"{key}_seed"] = np.array(seed)
            data[f"{key}_sha"] = np.array(digest(q, k, v, table))
            print(key, len(rows), "rows", file=sys.stderr)
    np.savez_compressed(OUT, **data)
    print(OUT, OUT.stat().st_size, "bytes")


def load_case(golden, hq, hkv, d, dt):
    """(q, k, v, table, rows, reference outputs [n_rows, G, D] float32) of one fixture case."""
    key = case_key(hq, hkv, d, dt)
    seed = int(golden[f"{key}_seed"])
    q, k, v, table = case_inputs(hq, hkv, d, dt, seed)
    if digest(q, k, v, table) != str(golden[f"{key}_sha"]):
        raise AssertionError(f"seeded inputs of {key} changed")
    rows = golden[f"{key}_rows"].astype(np.int64)
    if dt == "bfloat16":
        out = (golden[f"{key}_out_bf16bits"].astype(np.uint32) << 16).view(np.float32)
    else:
        out = golden[f"{key}_out"]
    return q, k, v, table, rows, out


if __name__ == "__main__":
    main()
