"""Decode metadata built on the device (b2a_decode_metadata) against the host builders.

The host path restates attention/metal.py:145-152 (page CSR from the host page
table, ``paged_kv_indices``) and cuts the split-KV plan with b2a_decode_plan.
The device path reads a device copy of the page table and must produce the
same integers, so decode through either gives the same bytes. The page-table
scatter that keeps the device copy current is checked against numpy.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import HeadConfig, rand, to_dev
from minisgl_b200 import workloads as W

pytestmark = pytest.mark.gpu

META_OVERFLOW = 34  # kWdMetaOverflow


def _device_error() -> int:
    import torch

    from minisgl_b200 import _native as nat

    code = ctypes.c_int(-1)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    return code.value


def _table(P: int, seed: int):
    """A fragmented pool's page table, its rows shuffled into a larger table with junk rows."""
    rng = np.random.default_rng(seed)
    lens = np.concatenate([[0, 1, P, P + 1, 3 * P, 700, 2049, 4096], rng.integers(1, 3000, 40)]).astype(np.int64)
    pb = W.allocate_pages(lens, 1 << 19, P, rng, max_seq_len=4096 + 64)
    R = len(lens) + 9
    table = rng.integers(0, 1 << 19, (R, pb.page_table.shape[1])).astype(np.int32)
    rows = rng.permutation(R)[: len(lens)].astype(np.int64)
    table[rows] = pb.page_table
    return table, rows, lens


def _device_meta(table, rows, lens, P, nc, idx_cap=None):
    import torch

    from minisgl_b200 import _native as nat

    B = len(lens)
    i32 = dict(dtype=torch.int32, device="cuda")
    d = dict(
        kv_indptr=torch.full((B + 1,), -7, **i32), kv_indices=torch.full((idx_cap or int(((lens + P - 1) // P).sum()) + 5,), -7, **i32),
        lpl=torch.full((B,), -7, **i32), cta=torch.full((nc + 1,), -7, **i32),
        segs=torch.full((B + nc + 1, 4), -7, **i32), merge=torch.full((B + 1,), -7, **i32),
        counts=torch.zeros(2, **i32),
    )
    t_dev = torch.from_numpy(table).cuda()
    r_dev = torch.from_numpy(rows.astype(np.int32)).cuda()
    l_dev = torch.from_numpy(lens.astype(np.int32)).cuda()
    nat.call("b2a_decode_metadata", t_dev.data_ptr(), table.shape[0], table.shape[1], r_dev.data_ptr(),
             l_dev.data_ptr(), B, P, nc, d["kv_indptr"].data_ptr(), d["kv_indices"].data_ptr(),
             d["kv_indices"].numel(), d["lpl"].data_ptr(), d["cta"].data_ptr(), d["segs"].data_ptr(),
             d["segs"].shape[0], d["merge"].data_ptr(), d["counts"].data_ptr(),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in d.items()}


@pytest.mark.parametrize("P", [1, 16])
@pytest.mark.parametrize("nc", [148, 7, 1])
def test_device_decode_metadata_matches_host(P, nc):
    from minisgl_b200 import _native as nat
    from minisgl_b200.attention.base import paged_kv_indices

    assert _device_error() == 0
    table, rows, lens = _table(P, seed=100 + P + nc)
    kv_indptr, kv_indices, lpl = paged_kv_indices(table, rows, lens, P)
    cta, segs, merge, n_part = nat.decode_plan(kv_indptr, lpl, P, nc)
    d = _device_meta(table, rows, lens, P, nc)
    total = int(kv_indptr[-1])
    assert np.array_equal(d["kv_indptr"], kv_indptr)
    assert np.array_equal(d["kv_indices"][:total], kv_indices)
    assert np.array_equal(d["lpl"], lpl)
    assert np.array_equal(d["cta"], cta)
    assert np.array_equal(d["segs"][: len(segs)], segs)
    assert np.array_equal(d["merge"], merge)
    assert d["counts"].tolist() == [len(segs), n_part]
    assert _device_error() == 0


def test_device_metadata_empty_and_single():
    from minisgl_b200 import _native as nat
    from minisgl_b200.attention.base import paged_kv_indices

    table = np.arange(64, dtype=np.int32).reshape(2, 32)
    for lens in (np.array([0, 0]), np.array([32, 0]), np.array([1, 1])):
        rows = np.array([1, 0])
        kv_indptr, kv_indices, lpl = paged_kv_indices(table, rows, lens, 1)
        cta, segs, merge, n_part = nat.decode_plan(kv_indptr, lpl, 1, 4)
        d = _device_meta(table, rows, lens, 1, 4)
        assert np.array_equal(d["kv_indptr"], kv_indptr) and np.array_equal(d["cta"], cta)
        assert np.array_equal(d["segs"][: len(segs)], segs) and np.array_equal(d["merge"], merge)
        assert np.array_equal(d["kv_indices"][: int(kv_indptr[-1])], kv_indices)


def test_decode_through_device_metadata_is_identical():
    """Same rows and lengths, metadata from the host or from the device: the same output bytes."""
    import torch

    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.kvcache import MHAKVCache

    rng = np.random.default_rng(5)
    lens = rng.integers(1, 2500, 37)
    pb = W.allocate_pages(lens, 1 << 17, 16, rng)
    kv = MHAKVCache(1, pb.num_slots, 8, 128, torch.bfloat16)
    kv.k[0].copy_(torch.from_numpy(rand(rng, (pb.num_slots, 8, 128), "bfloat16")))
    kv.v[0].copy_(torch.from_numpy(rand(rng, (pb.num_slots, 8, 128), "bfloat16")))
    be = B200AttnBackend(HeadConfig(16, 8, 128), kv, pb.page_table, page_size=16)
    B = len(lens)
    q = to_dev(rand(rng, (B, 16, 128), "bfloat16"), "bfloat16")
    host = be.alloc_decode_graph_metadata(B, int(((lens + 15) // 16).sum()))
    be.fill_decode_graph_metadata(host, pb.rows, lens)
    dev = be.alloc_decode_graph_metadata(B, int(((lens + 15) // 16).sum()))
    be.build_decode_metadata_device(dev, torch.from_numpy(pb.page_table).cuda(),
                                    torch.from_numpy(pb.rows.astype(np.int32)).cuda(),
                                    torch.from_numpy(lens.astype(np.int32)).cuda())
    a = be.forward_decode(q, 0, host)
    b = be.forward_decode(q, 0, dev)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_page_table_scatter():
    import torch

    from minisgl_b200.attention import page_table_scatter

    rng = np.random.default_rng(9)
    table = rng.integers(0, 1000, (12, 300)).astype(np.int32)
    t_dev = torch.from_numpy(table).cuda()
    n = 500
    r = rng.integers(0, 12, n).astype(np.int32)
    c = rng.permutation(12 * 300)[:n]  # distinct cells
    r, c = (c // 300).astype(np.int32), (c % 300).astype(np.int32)
    v = rng.integers(0, 1 << 20, n).astype(np.int32)
    page_table_scatter(t_dev, *(torch.from_numpy(x).cuda() for x in (r, c, v)))
    table[r, c] = v
    assert np.array_equal(t_dev.cpu().numpy(), table)


def test_out_of_range_rows_are_reported_and_skipped():
    import torch

    from minisgl_b200.attention import page_table_scatter

    assert _device_error() == 0
    table, rows, lens = _table(16, seed=3)
    bad = rows.copy()
    bad[4] = table.shape[0] + 5  # a row outside the table
    d = _device_meta(table, bad, lens, 16, 148)
    assert _device_error() == META_OVERFLOW
    assert np.all(d["kv_indices"][d["kv_indptr"][4]: d["kv_indptr"][5]] == -7)  # nothing written for it
    # scatter: an out-of-range column is dropped, the rest lands
    t_dev = torch.zeros((4, 8), dtype=torch.int32, device="cuda")
    page_table_scatter(t_dev, *(torch.tensor(x, dtype=torch.int32, device="cuda")
                                for x in ([0, 1, 2], [3, 9, 7], [11, 12, 13])))
    torch.cuda.synchronize()
    assert _device_error() == META_OVERFLOW
    want = np.zeros((4, 8), np.int32)
    want[0, 3], want[2, 7] = 11, 13
    assert np.array_equal(t_dev.cpu().numpy(), want)
    assert _device_error() == 0
