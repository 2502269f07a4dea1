"""Failure detection on the GPU without a GPU fault.

The kernels validate every page id and pool slot before they use it. A bad
one is never dereferenced: the access is skipped (decode completes its stage
on stale data, extend loads zeros through an out-of-range TMA coordinate, the
store drops the row) and the kernel records code 32 in the device watchdog
word, which b2a_device_error returns and clears. These tests plant such ids
on the host, check the code, and check that the context still produces
correct results afterwards.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import TOL, HeadConfig, max_abs, rand, to_dev, to_np
from minisgl_b200 import workloads as W
from oracle import attention as O

pytestmark = pytest.mark.gpu

BAD_SLOT = 32  # kWdBadSlot


def _device_error() -> int:
    import torch

    from minisgl_b200 import _native as nat

    code = ctypes.c_int(-1)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    return code.value


def _backend(pb, dtype="bfloat16", seed=0):
    import torch

    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.kvcache import MHAKVCache
    from helpers import torch_dtype

    rng = np.random.default_rng(seed)
    kv = MHAKVCache(1, pb.num_slots, 8, 128, torch_dtype(dtype))
    hk, hv = rand(rng, (pb.num_slots, 8, 128), dtype), rand(rng, (pb.num_slots, 8, 128), dtype)
    kv.k[0].copy_(torch.from_numpy(hk))
    kv.v[0].copy_(torch.from_numpy(hv))
    be = B200AttnBackend(HeadConfig(16, 8, 128), kv, pb.page_table, page_size=pb.page_size)
    return be, kv, hk, hv, rng


def test_decode_bad_page_is_reported_not_read():
    import torch

    assert _device_error() == 0
    rng = np.random.default_rng(1)
    lens = np.array([40, 100, 7, 300])
    pb = W.allocate_pages(lens, 4096, 16, rng)
    be, kv, hk, hv, rng = _backend(pb)
    good = pb.page_table.copy()
    pb.page_table[1, 16:32] = pb.num_slots + 64 + np.arange(16)  # request 1's second page: outside the pool
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens)
    q = rand(rng, (4, 16, 128), "bfloat16")
    be.forward_decode(to_dev(q, "bfloat16"), 0, meta)
    torch.cuda.synchronize()
    assert _device_error() == BAD_SLOT
    # the context is intact: the same call on a correct table is exact again
    pb.page_table[:] = good
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens)
    out = be.forward_decode(to_dev(q, "bfloat16"), 0, meta)
    torch.cuda.synchronize()
    idx, mask = O.naive_prepare_decode(pb.page_table, pb.rows, pb.lens)
    assert max_abs(to_np(out), O.naive_forward_decode(q, hk, hv, idx, mask, 128 ** -0.5)) <= TOL["bfloat16"]
    assert _device_error() == 0


def test_store_bad_slot_drops_only_that_row():
    import torch

    from minisgl_b200.config import RotaryConfig
    from minisgl_b200.kvcache import MHAKVCache
    from minisgl_b200.layers import RotaryEmbedding

    assert _device_error() == 0
    rng = np.random.default_rng(2)
    T, N = 6, 256
    q = to_dev(rand(rng, (T, 16, 128), "bfloat16"), "bfloat16")
    k = to_dev(rand(rng, (T, 8, 128), "bfloat16"), "bfloat16")
    v = to_dev(rand(rng, (T, 8, 128), "bfloat16"), "bfloat16")
    kv = MHAKVCache(1, N, 8, 128, torch.bfloat16)
    out_loc = np.array([3, 9, N + 5, 11, 200, 17], dtype=np.int32)  # token 2 points past the pool
    pos = np.arange(T, dtype=np.int32)
    rope = RotaryEmbedding(RotaryConfig(128, 128, 1e6, 4096))
    rope.rope_store_(q, k, v, torch.from_numpy(pos).cuda(), torch.from_numpy(out_loc).cuda(), kv, 0)
    torch.cuda.synchronize()
    assert _device_error() == BAD_SLOT
    good = [i for i in range(T) if out_loc[i] < N]
    assert np.array_equal(to_np(kv.v[0])[out_loc[good]], to_np(v)[good])
    assert np.array_equal(to_np(kv.k[0])[out_loc[good]], to_np(k)[good])
    untouched = np.setdiff1d(np.arange(N), out_loc[good])
    assert not to_np(kv.k[0])[untouched].any() and not to_np(kv.v[0])[untouched].any()


@pytest.mark.parametrize("P", [16, 1])
def test_extend_bad_page_is_reported_not_read(P):
    """tcgen05 extend (P=16) and the packed small-page path (P=1)."""
    import torch

    assert _device_error() == 0
    eb = W.config3_batch(seed=3, batch=4, page_size=P)
    pb = eb.paged
    be, kv, hk, hv, rng = _backend(pb)
    good = pb.page_table.copy()
    pb.page_table[0, 32:48] = pb.num_slots + 4096 + np.arange(16)  # inside request 0's prefix
    meta = be.extend_metadata_from_lens(pb.rows, pb.lens, eb.extend)
    T = int(eb.extend.sum())
    q = to_dev(rand(rng, (T, 16, 128), "bfloat16"), "bfloat16")
    be._forward_prefill(q, None, None, 0, meta)
    torch.cuda.synchronize()
    assert _device_error() == BAD_SLOT
    pb.page_table[:] = good
    meta = be.extend_metadata_from_lens(pb.rows, pb.lens, eb.extend)
    out = be._forward_prefill(q, None, None, 0, meta)
    torch.cuda.synchronize()
    assert _device_error() == 0
    assert np.isfinite(to_np(out)).all()


BAD_PLAN = 35  # kWdBadPlan


@pytest.mark.parametrize("field", ["slot", "request"])
def test_decode_bad_plan_segment_is_skipped_and_reported(field):
    """A plan whose segment names a partial slot past the workspace, or a request past B,
    is never followed: the segment is skipped (no partial row or output row is written
    through it) and code 35 is reported. The workspace is then zeroed again (a skipped
    segment leaves its request's merge counter short) and a correct plan is exact."""
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.attention.base import paged_kv_indices

    assert _device_error() == 0
    rng = np.random.default_rng(5)
    lens = rng.integers(200, 3000, size=9)
    pb = W.allocate_pages(lens, 65536, 16, rng)
    be, kv, hk, hv, rng = _backend(pb)
    ind, idx, lpl = paged_kv_indices(pb.page_table, pb.rows, pb.lens, 16)
    nc = 64
    cta, segs, merge, n_part = nat.decode_plan(ind, lpl, 16, nc)
    split = np.nonzero(segs[:, 3] >= 0)[0]
    assert split.size >= 2
    bad = segs.copy()
    if field == "slot":
        bad[split[0], 3] = n_part + 5
    else:
        bad[split[0], 0] = len(lens) + 3
    q = rand(rng, (len(lens), 16, 128), "bfloat16")
    qd = to_dev(q, "bfloat16")
    ws_bytes = nat.decode_workspace_bytes(n_part, 16, 128)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.zeros_like(qd)
    stream = torch.cuda.current_stream().cuda_stream

    def call(plan):
        dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (idx, cta, plan, merge)]
        nat.call("b2a_decode", qd.data_ptr(), kv.k[0].data_ptr(), kv.v[0].data_ptr(), pb.num_slots,
                 dev[0].data_ptr(), 16, dev[1].data_ptr(), dev[2].data_ptr(), nc, dev[3].data_ptr(), n_part,
                 len(lens), 16, 8, 128, float(128 ** -0.5), ws.data_ptr(), ws_bytes, out.data_ptr(),
                 nat.B2A_DTYPE_BF16, stream)
        torch.cuda.synchronize()

    call(bad)
    assert _device_error() == BAD_PLAN
    ws.zero_()
    call(segs)
    assert _device_error() == 0
    gidx, mask = O.naive_prepare_decode(pb.page_table, pb.rows, pb.lens)
    assert max_abs(to_np(out), O.naive_forward_decode(q, hk, hv, gidx, mask, 128 ** -0.5)) <= TOL["bfloat16"]
