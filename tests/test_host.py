"""CPU tests of the host side: metadata builders, plans, the C ABI surface.

No GPU work is launched here; the plan functions of libb200attn.so are pure
host code and the library loads without a driver.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest

from minisgl_b200 import _native as nat
from minisgl_b200 import workloads as W
from minisgl_b200.attention.base import paged_kv_indices
from minisgl_b200.layers import llama3_freqs, rope_tables
from minisgl_b200.config import RotaryConfig
from oracle import attention as O

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200attn.h"


def test_library_exports_every_declared_symbol():
    decls = re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(b2a_\w+)\s*\(", HEADER.read_text(), re.M)
    assert len(decls) >= 12
    for name in decls:
        assert hasattr(nat.LIB, name), f"{name} declared in b200attn.h but not exported"
    assert set(decls) == set(nat.SIGNATURES), "ctypes table and header disagree"
    assert nat.LIB.b2a_abi_version() == 1


def _table_and_lens(seed=0, B=9, P=16, num_slots=8192):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 700, size=B)
    lens[0] = 1
    lens[1] = P
    lens[2] = P + 1
    return W.allocate_pages(lens, num_slots, P, rng)


def test_page_size_1_indices_equal_metal_csr():
    """attention/metal.py:145-152 restated by the oracle == the backend's builder, bit-exact."""
    pb = W.config1_batch(seed=3)
    ind, idx, lpl = paged_kv_indices(pb.page_table, pb.rows, pb.lens, 1)
    ref_ptr, ref_idx = O.metal_prepare_decode(pb.page_table, pb.rows, pb.lens)
    np.testing.assert_array_equal(ind, ref_ptr)
    np.testing.assert_array_equal(idx, ref_idx)
    assert (lpl == 1).all()


@pytest.mark.parametrize("P", [2, 4, 16, 64])
def test_paged_indices_expand_to_page_table_slots(P):
    """Expanding page ids back to slots reproduces page_table[row, :len] exactly."""
    pb = _table_and_lens(P=P, num_slots=P * 2048)
    ind, idx, lpl = paged_kv_indices(pb.page_table, pb.rows, pb.lens, P, check=True)
    for b in range(pb.batch_size):
        pages = idx[ind[b]:ind[b + 1]].astype(np.int64)
        n = int(pb.lens[b])
        slots = (pages[:, None] * P + np.arange(P)[None]).reshape(-1)[:n]
        np.testing.assert_array_equal(slots, pb.page_table[b, :n])
        assert lpl[b] == n - (len(pages) - 1) * P


def test_paged_indices_reject_non_contiguous_pages():
    pb = _table_and_lens(P=4, num_slots=4096)
    pb.page_table[3, 1] += 1
    with pytest.raises(ValueError):
        paged_kv_indices(pb.page_table, pb.rows, pb.lens, 4, check=True)


@pytest.mark.parametrize("num_ctas", [1, 3, 8, 148, 1000])
@pytest.mark.parametrize("P", [1, 16])
def test_decode_plan_covers_every_page_once(num_ctas, P):
    pb = _table_and_lens(P=P, num_slots=P * 4096) if P > 1 else W.config1_batch(seed=1)
    ind, idx, lpl = paged_kv_indices(pb.page_table, pb.rows, pb.lens, P)
    cta_indptr, segs, merge_indptr, n_part = nat.decode_plan(ind, lpl, P, num_ctas)
    B = pb.batch_size
    assert cta_indptr[0] == 0 and cta_indptr[-1] == len(segs)
    assert (np.diff(cta_indptr) >= 0).all()
    covered = {b: 0 for b in range(B)}
    slots_seen = []
    for b, pbeg, ntok, slot in segs.tolist():
        covered[b] += ntok
        slots_seen.append(slot)
        assert ind[b] <= pbeg < ind[b + 1] or ntok == 0
    for b in range(B):
        assert covered[b] == pb.lens[b]
        n = merge_indptr[b + 1] - merge_indptr[b]
        pieces = sum(1 for s in segs.tolist() if s[0] == b)
        assert n == (pieces if pieces > 1 else 0)
    used = [s for s in slots_seen if s >= 0]
    assert sorted(used) == list(range(n_part))
    # balance: no CTA holds more than ceil(total/num_ctas) pages, or 64 tokens' worth
    per = max(-(-int(ind[-1]) // num_ctas), max(1, 64 // P))
    for c in range(num_ctas):
        pages = 0
        for b, pbeg, ntok, _ in segs[cta_indptr[c]:cta_indptr[c + 1]].tolist():
            pages += -(-ntok // P)
        assert pages <= per + 1


@pytest.mark.parametrize("P", [1, 16])
def test_decode_plan_minimum_share_for_tiny_batches(P):
    """A CTA's share is at least 64 tokens' worth of pages: one request of 1024 tokens over
    148 CTAs becomes 1024 / 64 = 16 pieces (not one partial per page); a batch large enough
    for 148 shares of 64 tokens is cut as before."""
    pages = 1024 // P
    ind = np.array([0, pages], np.int32)
    cta_indptr, segs, merge_indptr, n_part = nat.decode_plan(ind, None, P, 148)
    assert n_part == 16 and len(segs) == 16
    assert (np.diff(cta_indptr)[:16] == 1).all() and (np.diff(cta_indptr)[16:] == 0).all()
    assert all(ntok == 64 for _, _, ntok, _ in segs.tolist())
    big = 148 * 2 * 64 // P  # two minimum shares per CTA
    cta_indptr, segs, _, n_part = nat.decode_plan(np.array([0, big], np.int32), None, P, 148)
    assert len(segs) == 148 and n_part == 148


def test_decode_plan_rejects_bad_input():
    with pytest.raises(ValueError, match="monotonic"):
        nat.decode_plan(np.array([0, 5, 3], np.int32), None, 1, 4)
    with pytest.raises(ValueError, match="power of two"):
        nat.decode_plan(np.array([0, 5], np.int32), None, 3, 4)
    with pytest.raises(ValueError, match="last_page_len"):
        nat.decode_plan(np.array([0, 2], np.int32), np.array([17], np.int32), 16, 4)


def test_extend_plan_tiles_and_order():
    eb = W.config3_batch(seed=0)
    P = eb.paged.page_size
    ind, idx, lpl = paged_kv_indices(eb.paged.page_table, eb.paged.rows, eb.paged.lens, P)
    qo = np.concatenate([[0], np.cumsum(eb.extend)]).astype(np.int32)
    work = nat.extend_plan(qo, ind, lpl, P, 64)
    rows = {}
    for r, tb, nq, _ in work.tolist():
        assert 0 < nq <= 64 and tb % 64 == 0
        rows[r] = rows.get(r, 0) + nq
    assert rows == {r: int(e) for r, e in enumerate(eb.extend)}
    cost = [nq * (int(eb.prefix[r]) + tb + nq) for r, tb, nq, _ in work.tolist()]
    assert cost == sorted(cost, reverse=True)
    with pytest.raises(ValueError, match="kv length"):
        nat.extend_plan(np.array([0, 40], np.int32), np.array([0, 1], np.int32), np.array([8], np.int32), 16, 64)


def test_rope_tables():
    inv, s = rope_tables(RotaryConfig(128, 128, 1e6, 40960))
    np.testing.assert_allclose(inv, O.rope_inv_freq(128, 1e6), rtol=0)
    assert s == 1.0
    inv, s = rope_tables(RotaryConfig(128, 128, 1e4, 4096, {"rope_type": "linear", "factor": 4.0}))
    assert s == 0.25
    cfg = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
           "original_max_position_embeddings": 8192}
    inv, s = rope_tables(RotaryConfig(128, 128, 5e5, 131072, cfg))
    np.testing.assert_allclose(inv, (1.0 / llama3_freqs(128, 5e5, cfg)).astype(np.float32))
    # high-frequency dims untouched, low-frequency dims slowed by `factor`
    plain = O.rope_inv_freq(128, 5e5)
    assert inv[0] == plain[0]
    np.testing.assert_allclose(inv[-1], plain[-1] / 8.0, rtol=1e-6)
    with pytest.raises(NotImplementedError):
        rope_tables(RotaryConfig(128, 128, 1e4, 4096, {"rope_type": "yarn", "factor": 2.0}))


def test_registry_rejects_unknown_backend():
    from minisgl_b200.attention import SUPPORTED_ATTENTION_BACKENDS, create_attention_backend

    assert list(SUPPORTED_ATTENTION_BACKENDS) == ["b200"]
    with pytest.raises(ValueError, match="Unknown attention backend 'metal'"):
        create_attention_backend("metal", None, None, None)


def test_shard_requests_partitions_and_balances():
    lens = W.config5_lens(seed=0, batch=257)
    for world in (1, 2, 4, 8):
        shards = W.shard_requests(lens, world)
        allids = np.sort(np.concatenate(shards))
        np.testing.assert_array_equal(allids, np.arange(257))
        loads = [lens[s].sum() for s in shards]
        assert max(loads) <= (sum(loads) / world) + lens.max()


def test_workload_generators_are_seeded_and_valid():
    a, b = W.config2_batch(seed=5, batch=16), W.config2_batch(seed=5, batch=16)
    np.testing.assert_array_equal(a.page_table, b.page_table)
    ind, idx, lpl = paged_kv_indices(a.page_table, a.rows, a.lens, 16, check=True)
    assert len(np.unique(idx)) == len(idx)  # pages are never shared
    eb = W.config3_batch(seed=0)
    assert eb.prefix[0] % 16 != 0 or eb.prefix[0] == 0
    assert all(p % 16 == 0 for p in eb.prefix[1:])
    assert (eb.extend >= 64).all() and (eb.extend <= 512).all()


def test_swiglu_rejects_bad_sizes_before_any_launch():
    # argument checks return before any CUDA call, so they run without a GPU
    dummy = 16  # never dereferenced: every call below fails or returns before a launch
    with pytest.raises(ValueError, match="even"):
        nat.call("b2a_swiglu", dummy, 8, dummy, 4, 3, nat.B2A_DTYPE_BF16, None)
    with pytest.raises(ValueError, match="row_stride"):
        nat.call("b2a_swiglu", dummy, 6, dummy, 4, 4, nat.B2A_DTYPE_BF16, None)
    with pytest.raises(ValueError, match="negative"):
        nat.call("b2a_swiglu", dummy, 8, dummy, -1, 4, nat.B2A_DTYPE_BF16, None)
    nat.call("b2a_swiglu", dummy, 8, dummy, 0, 4, nat.B2A_DTYPE_BF16, None)  # nothing to do


def test_proj_rejects_bad_arguments_before_any_launch():
    dummy = 16  # never dereferenced: every call below fails or returns before a launch
    bf16 = nat.B2A_DTYPE_BF16

    def call(M=4, K=1024, N=1024, mode=0, dtype=bf16, x_stride=1024, res=0, out_stride=1024):
        nat.call("b2a_proj", dummy, x_stride, M, K, dummy, N, 0, 1e-6, res, 1024, dummy, out_stride, mode,
                 dtype, None)

    with pytest.raises(nat.B200AttnError, match="at most 64"):
        call(M=65)
    with pytest.raises(nat.B200AttnError, match="multiple of 128"):
        call(K=1000, x_stride=1000)
    with pytest.raises(nat.B200AttnError, match="multiple of 16"):
        call(N=1000)
    with pytest.raises(nat.B200AttnError, match="multiple of 32"):
        call(N=1040, mode=2)
    with pytest.raises(nat.B200AttnError, match="bf16 only"):
        call(dtype=nat.B2A_DTYPE_F32)
    with pytest.raises(ValueError, match="unknown proj mode"):
        call(mode=3)
    with pytest.raises(ValueError, match="NULL"):
        call(mode=1)  # residual without res
    with pytest.raises(ValueError, match="x_row_stride"):
        call(x_stride=1020)
    with pytest.raises(ValueError, match="negative"):
        call(M=-1)
    call(M=0)  # nothing to do


def test_extend_executed_flops_counts_whole_tiles_and_blocks():
    """bench.extend_executed_flops against a brute-force walk of the tcgen05 kernel's
    work: items of two 128/G-token tiles, each over whole 128-key blocks up to the last
    key its last row sees; never less than the visible-key FLOPs."""
    import bench

    rng = np.random.default_rng(2)
    Hq, Hkv, D = 16, 8, 128
    G = Hq // Hkv
    prefix = rng.integers(0, 700, 9) // 16 * 16
    extend = rng.integers(1, 400, 9)
    blocks = 0
    for p, e in zip(prefix, extend):
        for tok0 in range(0, int(e), 2 * (128 // G)):
            for t in range(2):
                first = tok0 + t * (128 // G)
                last = min(int(e), first + 128 // G) - 1
                if last < first:
                    continue
                keys = int(p) + last + 1  # keys visible to the tile's last row
                blocks += -(-keys // 128)
    want = blocks * Hkv * 2 * (2 * 128 * 128 * D)
    got = bench.extend_executed_flops(prefix, extend, Hq, Hkv, D)
    assert got == want
    assert got >= bench.extend_flops(prefix, extend, Hq, D)
