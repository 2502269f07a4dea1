"""Golden vectors from the reference's own kernel.

tests/golden/paged_decode_metal_ref.npz holds the outputs of the reference's
Metal paged-decode kernel body (python/minisgl_mlx/attention/metal.py:35-95),
executed on the CPU by oracle/metal_ref, on the reference test's case list
(tests/test_attention.py:19-32). Generator: tests/golden/make_golden.py.

* CPU: the seeded inputs still hash to what the fixture was made from, the
  numpy oracle agrees with the reference kernel's outputs (this pins the
  oracle), and -- where the reference checkout is present -- re-running the
  kernel reproduces the fixture bit for bit.
* GPU: both CUDA decode entry points agree with the reference kernel's outputs, and so
  does extend attention with one new token per request (the single-query case of the
  prefill path), on the SIMT and the tcgen05 kernels.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

from make_golden import DTYPES, SHAPES, case_inputs, case_key, digest  # noqa: E402

from helpers import TOL, max_abs, to_dev, to_np  # noqa: E402
from oracle import attention as O  # noqa: E402

FIXTURE = Path(__file__).resolve().parent / "golden" / "paged_decode_metal_ref.npz"
CASES = [(hq, hkv, d, dt) for (hq, hkv, d) in SHAPES for dt in DTYPES]


@pytest.fixture(scope="module")
def golden():
    return np.load(FIXTURE)


def _case(golden, hq, hkv, d, dt):
    key = case_key(hq, hkv, d, dt)
    seed = int(golden[f"{key}_seed"])
    q, k, v, indptr, idx, per = case_inputs(hq, hkv, d, dt, seed)
    assert digest(q, k, v, indptr, idx) == str(golden[f"{key}_sha"]), "seeded inputs changed"
    return q, k, v, indptr, idx, per, golden[f"{key}_out"]


@pytest.mark.parametrize("hq,hkv,d,dt", CASES)
def test_oracle_matches_reference_kernel(golden, hq, hkv, d, dt):
    q, k, v, indptr, idx, per, ref_out = _case(golden, hq, hkv, d, dt)
    oracle = O.reference_decode_per_request(q, k, v, per, d ** -0.5)
    # the reference kernel rounds its output to the input dtype
    assert max_abs(oracle, ref_out) <= TOL[dt]
    if dt == "float32":
        assert max_abs(oracle, ref_out) <= 2e-6


def test_reference_kernel_reproduces_fixture(golden):
    from oracle import metal_ref

    if not metal_ref.available():
        pytest.skip("oracle/_ref/libmetal_ref.so not built (needs the reference checkout)")
    hq, hkv, d, dt = CASES[1]
    q, k, v, indptr, idx, _, ref_out = _case(golden, hq, hkv, d, dt)
    again = metal_ref.metal_paged_decode(q, k, v, indptr, idx, d ** -0.5, dt)
    np.testing.assert_array_equal(again, ref_out)


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv,d,dt", CASES)
def test_cuda_decode_matches_reference_kernel(golden, hq, hkv, d, dt):
    import torch

    from minisgl_b200.attention import paged_decode_attention

    q, k, v, indptr, idx, per, ref_out = _case(golden, hq, hkv, d, dt)
    out = paged_decode_attention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), torch.from_numpy(indptr).cuda(),
                                 torch.from_numpy(idx).cuda(), d ** -0.5)
    torch.cuda.synchronize()
    assert max_abs(to_np(out), ref_out) <= TOL[dt]


@pytest.mark.gpu
@pytest.mark.parametrize("hq,hkv,d,dt", CASES)
def test_cuda_extend_single_query_matches_reference_kernel(golden, hq, hkv, d, dt):
    """With one new token per request, extend attention over the L - 1 cached tokens plus the
    token itself (bottom-right causal) is the decode the reference's Metal kernel computed.
    The backend's prefill path at page size 1 -- the SIMT kernel, or for bf16 with D = 128
    the page packer and the tcgen05 kernel -- must reproduce the golden outputs."""
    import torch

    from helpers import torch_dtype
    from minisgl_b200 import MHAKVCache
    from minisgl_b200.attention import B200AttnBackend

    q, k, v, indptr, idx, per, ref_out = _case(golden, hq, hkv, d, dt)
    B = len(indptr) - 1
    lens = np.diff(indptr).astype(np.int64)
    table = np.zeros((B, int(lens.max())), np.int32)
    for b in range(B):
        table[b, : lens[b]] = idx[indptr[b]: indptr[b + 1]]

    class Cfg:
        num_qo_heads, num_kv_heads, head_dim = hq, hkv, d

    kv = MHAKVCache(1, k.shape[0], hkv, d, torch_dtype(dt))
    kv.k[0].copy_(to_dev(k, dt))
    kv.v[0].copy_(to_dev(v, dt))
    be = B200AttnBackend(Cfg, kv, table, page_size=1)
    meta = be.extend_metadata_from_lens(np.arange(B), lens, np.ones(B, np.int64))
    out = be._forward_prefill(to_dev(q, dt), None, None, 0, meta)
    torch.cuda.synchronize()
    assert max_abs(to_np(out), ref_out) <= TOL[dt]
