"""The allocation-free decode entry point (b2a_decode_noalloc).

Some callers cannot allocate device memory when decode runs -- an engine
whose memory planner gave the device to the KV pool, or a host that may only
hand over buffers it already owns. For them b2a_decode_noalloc keeps the
split-KV partials and merge counters in a static device array of the library.
This test calls it through the C ABI twice in a row (the second call reuses the
array with the first call's contents still in it) and checks each result
against the CPU oracle (the reference's naive decode restated in float64) and
against the workspace-taking b2a_decode on the same inputs.

The file name sorts last so that a stop-at-first-failure run has executed
every other test before this one; it also passes on its own in a fresh
process.
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import TOL, max_abs, rand, to_dev, to_np
from oracle import attention as O

pytestmark = pytest.mark.gpu


def _decode_both(dtype: str, P: int, seed: int):
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200 import workloads as W
    from minisgl_b200.attention.base import paged_kv_indices
    from minisgl_b200.kvcache.pool import dtype_code

    Hq, Hkv, D, N = 16, 8, 128, 65536
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 3000, size=37)
    pb = W.allocate_pages(lens, N, P, rng)
    hk, hv = rand(rng, (N, Hkv, D), dtype), rand(rng, (N, Hkv, D), dtype)
    hq = rand(rng, (len(lens), Hq, D), dtype)
    kp, vp, q = to_dev(hk, dtype), to_dev(hv, dtype), to_dev(hq, dtype)
    ind, idx, lpl = paged_kv_indices(pb.page_table, pb.rows, pb.lens, P)
    num_ctas = 148  # cuts most requests so the split partials and their merge are exercised
    cta_indptr, segs, merge_indptr, n_part = nat.decode_plan(ind, lpl, P, num_ctas)
    assert n_part > 0
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (idx, cta_indptr, segs, merge_indptr)]
    stream = torch.cuda.current_stream().cuda_stream
    code = dtype_code(kp.dtype)
    ws_bytes = nat.decode_workspace_bytes(n_part, Hq, D)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")  # merge counters start at zero
    ref = torch.empty_like(q)
    nat.call("b2a_decode", q.data_ptr(), kp.data_ptr(), vp.data_ptr(), N, dev[0].data_ptr(), P,
             dev[1].data_ptr(), dev[2].data_ptr(), num_ctas, dev[3].data_ptr(), n_part, len(lens), Hq, Hkv,
             D, float(D ** -0.5), ws.data_ptr(), ws_bytes, ref.data_ptr(), code, stream)
    out = torch.empty_like(q)
    nat.call("b2a_decode_noalloc", q.data_ptr(), kp.data_ptr(), vp.data_ptr(), N, dev[0].data_ptr(), P,
             dev[1].data_ptr(), dev[2].data_ptr(), num_ctas, dev[3].data_ptr(), n_part, len(lens), Hq, Hkv,
             D, float(D ** -0.5), out.data_ptr(), code, stream)
    torch.cuda.synchronize()
    # the reference's naive decode (attention/naive.py:36-60) in float64
    gidx, mask = O.naive_prepare_decode(pb.page_table, pb.rows, pb.lens)
    oracle = O.naive_forward_decode(hq, hk, hv, gidx, mask, D ** -0.5)
    return to_np(out), to_np(ref), oracle


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_noalloc_decode_matches_oracle_and_workspace_decode_twice(dtype):
    # two calls in a row with different inputs: the shared scratch keeps the first
    # call's partials and counters, which must not leak into the second result
    for seed, P in ((0, 16), (1, 1)):
        out, ref, oracle = _decode_both(dtype, P, seed)
        assert max_abs(out, oracle) <= TOL[dtype], (seed, P, max_abs(out, oracle))
        assert max_abs(ref, oracle) <= TOL[dtype], (seed, P, max_abs(ref, oracle))
        assert max_abs(out, ref) <= TOL[dtype], (seed, P, max_abs(out, ref))


def test_noalloc_rejects_plans_larger_than_the_static_scratch():
    import ctypes

    import torch

    from minisgl_b200 import _native as nat

    Hq, D = 64, 256
    too_many = (8 << 20) // (Hq * (D + 2) * 4) + 1
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(nat.B200AttnError, match="static scratch"):
        nat.call("b2a_decode_noalloc", dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 1, dummy.data_ptr(), 1,
                 dummy.data_ptr(), dummy.data_ptr(), 1, dummy.data_ptr(), too_many, 1, Hq, 8, D, 1.0,
                 dummy.data_ptr(), nat.B2A_DTYPE_BF16, torch.cuda.current_stream().cuda_stream)
    code = ctypes.c_int(-1)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert code.value == 0
