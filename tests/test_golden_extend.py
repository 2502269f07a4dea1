"""Multi-query causal extend pinned to vectors made by the reference's own kernel.

tests/golden/extend_metal_ref.npz holds, for a ragged 10-request extend batch
(extend lengths 1, 2, 17, 127, 128, 129, 300, 64, 33, 5 over prefixes 0, 5, 33,
100, 16, 250, 3, 48, 0, 1000), the outputs of sampled causal query rows. Each
row i of request r attends keys [0, P_r + i], the bottom-right causal rule of the
reference's prefill (python/minisgl_mlx/attention/base.py:85-105); the fixture
computed that decode with the reference's Metal kernel body
(python/minisgl_mlx/attention/metal.py:35-95) run on the CPU by oracle/metal_ref.
Generator: tests/golden/make_golden_extend.py.

* CPU: the seeded inputs still hash to the fixture's, the float64 oracle of the
  reference's prefill (oracle.attention.forward_prefill) agrees with the
  reference kernel on every stored row (this pins the oracle for multi-query
  extend), and -- where the reference checkout was built -- re-running the kernel
  reproduces stored rows bit for bit.
* GPU: the backend's prefill path reproduces the stored rows at page size 16 (the
  tcgen05 kernel for bf16, the SIMT kernel for fp32) and at page size 1 (the tcgen05
  kernel over 16-key groups for bf16, the SIMT kernel for fp32).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

import make_golden_extend as GE  # noqa: E402

from helpers import TOL, HeadConfig, max_abs, to_dev, to_np  # noqa: E402
from oracle import attention as O  # noqa: E402

FIXTURE = Path(__file__).resolve().parent / "golden" / "extend_metal_ref.npz"
CASES = [(hq, hkv, d, dt) for (hq, hkv, d) in GE.SHAPES for dt in GE.DTYPES]


@pytest.fixture(scope="module")
def golden():
    return np.load(FIXTURE)


def _stored(out: np.ndarray, rows: np.ndarray, G: int) -> np.ndarray:
    """out [T, Hq, D] -> the stored rows' [n, G, D] (all G query heads of the row's kv head)."""
    return np.stack([out[t, h * G:(h + 1) * G] for t, h in zip(rows[:, 0], rows[:, 3])])


def _oracle_all_rows(q, k, v, table):
    lens = np.array(GE.PREFIX) + np.array(GE.EXTEND)
    meta = O.prepare_prefill(table, np.arange(len(lens)), GE.PREFIX, lens)
    T = q.shape[0]
    # no request reads fresh rows here: the pool already holds every key (prefix 0 included),
    # so the pool branch is taken for all of them
    meta.kv_indices = [table[r, :n].copy() for r, n in enumerate(lens)]
    return O.forward_prefill(q, None, None, k, v, meta, q.shape[2] ** -0.5)


def test_fixture_covers_the_causal_cases(golden):
    rows = golden["16_8_128_float32_rows"]
    # every request is present, with its first and last row
    for r, E in enumerate(GE.EXTEND):
        mine = rows[rows[:, 1] == r]
        assert mine[:, 2].min() == 0 and mine[:, 2].max() == E - 1
    assert set(rows[:, 3].tolist()) == set(range(8))


@pytest.mark.parametrize("hq,hkv,d,dt", CASES)
def test_oracle_matches_reference_kernel_extend(golden, hq, hkv, d, dt):
    q, k, v, table, rows, ref = GE.load_case(golden, hq, hkv, d, dt)
    oracle = _stored(_oracle_all_rows(q, k, v, table), rows, hq // hkv)
    assert max_abs(oracle, ref) <= TOL[dt]
    if dt == "float32":
        assert max_abs(oracle, ref) <= 2e-6


def test_reference_kernel_reproduces_extend_fixture(golden):
    from oracle import metal_ref

    if not metal_ref.available():
        pytest.skip("oracle/_ref/libmetal_ref.so not built (needs the reference checkout)")
    hq, hkv, d, dt = CASES[1]
    q, k, v, table, rows, ref = GE.load_case(golden, hq, hkv, d, dt)
    pick = np.nonzero(rows[:, 1] != 6)[0][::3]  # a third of the rows outside the longest request
    again = GE.run_reference_rows(q, k, v, table, hq, hkv, d, dt, rows[pick])
    np.testing.assert_array_equal(again, ref[pick])


@pytest.mark.gpu
@pytest.mark.parametrize("P", [16, 1])
@pytest.mark.parametrize("hq,hkv,d,dt", CASES)
def test_cuda_extend_matches_reference_kernel(golden, hq, hkv, d, dt, P):
    import torch

    from helpers import torch_dtype
    from minisgl_b200 import MHAKVCache
    from minisgl_b200 import _native as nat
    from minisgl_b200.attention import B200AttnBackend

    q, k, v, table, rows, ref = GE.load_case(golden, hq, hkv, d, dt)
    kv = MHAKVCache(1, k.shape[0], hkv, d, torch_dtype(dt))
    kv.k[0].copy_(to_dev(k, dt))
    kv.v[0].copy_(to_dev(v, dt))
    be = B200AttnBackend(HeadConfig(hq, hkv, d), kv, table, page_size=P)
    lens = np.array(GE.PREFIX) + np.array(GE.EXTEND)
    meta = be.extend_metadata_from_lens(np.arange(len(lens)), lens, np.array(GE.EXTEND))
    if dt == "bfloat16":  # the tensor-core kernel (over 16-key groups at page size 1)
        assert nat.extend_tile_q(hq, hkv, d, nat.B2A_DTYPE_BF16, 16) == 2 * 128 // (hq // hkv)
        assert meta.group_starts == (P == 1)
    out = be._forward_prefill(to_dev(q, dt), None, None, 0, meta)
    torch.cuda.synchronize()
    got = _stored(to_np(out), rows, hq // hkv)
    assert max_abs(got, ref) <= TOL[dt], max_abs(got, ref)
