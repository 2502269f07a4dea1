"""GPU parity of ragged causal extend (prefill) attention against the oracle.

The oracle is the reference's shared prefill (attention/base.py:70-105): per
request SDPA, fresh k/v when nothing is cached, the pool rows of
page_table[row, :device_len] otherwise, causal bottom-right when Lq > 1.
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import TOL, HeadConfig, max_abs, rand, to_dev, to_np, torch_dtype
from minisgl_b200 import workloads as W
from oracle import attention as O

pytestmark = pytest.mark.gpu


def _run_extend(eb: W.ExtendBatch, Hq, Hkv, D, dtype, seed=0):
    pb = eb.paged
    rng = np.random.default_rng(seed)
    N = pb.num_slots
    hk = rand(rng, (N, Hkv, D), dtype)
    hv = rand(rng, (N, Hkv, D), dtype)
    q = rand(rng, (int(eb.extend.sum()), Hq, D), dtype)
    return _run_extend_arrays(eb, Hq, Hkv, D, dtype, hk, hv, q)


def _run_extend_arrays(eb: W.ExtendBatch, Hq, Hkv, D, dtype, hk, hv, q):
    import torch

    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.kvcache import MHAKVCache

    pb = eb.paged
    N = pb.num_slots
    kv = MHAKVCache(1, N, Hkv, D, torch_dtype(dtype))
    kv.k[0].copy_(torch.from_numpy(hk))
    kv.v[0].copy_(torch.from_numpy(hv))
    be = B200AttnBackend(HeadConfig(Hq, Hkv, D), kv, pb.page_table, page_size=pb.page_size)
    meta = be.extend_metadata_from_lens(pb.rows, pb.lens, eb.extend)
    out = be._forward_prefill(to_dev(q, dtype), None, None, 0, meta)
    torch.cuda.synchronize()
    # oracle: fresh k/v rows are the pool rows just stored at positions [prefix, len)
    ks, vs = [], []
    for b in range(pb.batch_size):
        sl = pb.page_table[b, int(eb.prefix[b]):int(pb.lens[b])]
        ks.append(hk[sl])
        vs.append(hv[sl])
    omet = O.prepare_prefill(pb.page_table, pb.rows, eb.prefix, pb.lens)
    ref = O.forward_prefill(q, np.concatenate(ks), np.concatenate(vs), hk, hv, omet, D ** -0.5)
    np.testing.assert_array_equal(to_np(meta.last_indices).astype(np.int64), omet.last_indices)
    return to_np(out), ref


def _batch(prefix, extend, P, seed=0, slots=None):
    rng = np.random.default_rng(seed)
    prefix = np.asarray(prefix, np.int64)
    extend = np.asarray(extend, np.int64)
    lens = prefix + extend
    n = slots or int(((lens + P - 1) // P * P).sum() * 2 + 4 * P)
    pb = W.allocate_pages(lens, n // P * P, P, rng)
    return W.ExtendBatch(pb, prefix, extend)


EDGE = dict(prefix=[0, 0, 5, 16, 100, 31, 700, 0], extend=[1, 7, 1, 64, 130, 2, 65, 200])


@pytest.mark.parametrize("hq,hkv,d", [(16, 8, 128), (32, 8, 128), (8, 8, 64), (16, 2, 256)])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("P", [1, 16])
def test_extend_edge_cases(hq, hkv, d, dtype, P):
    eb = _batch(EDGE["prefix"], EDGE["extend"], P, seed=1)
    out, ref = _run_extend(eb, hq, hkv, d, dtype, seed=2)
    err = max_abs(out, ref)
    assert err <= TOL[dtype], err


def _max_jumps(s2: np.ndarray, block: int = 128) -> list:
    """How far each 128-key block's max rises above the running max before it, in log2
    units, for one query row whose visible scores (s * scale * log2 e) are s2: the factor
    2^-jump by which the tcgen05 extend rescales O and the row sum when a jump passes 8."""
    jumps, m = [], float(s2[:block].max())
    for j in range(1, -(-len(s2) // block)):
        mb = float(s2[j * block:(j + 1) * block].max())
        jumps.append(mb - m)
        m = max(m, mb)
    return jumps


def test_extend_score_jumps_across_key_blocks():
    """bf16 tcgen05 extend with planted key spikes that make a later key block score far
    above the earlier ones, so that O and the row sum are rescaled by 2^-33, by 2^-16 then
    2^-49, and by a factor below fp32's normal range (2^-130, which flushes the earlier terms to zero),
    against the float64 oracle. q is all ones and every head of a spike key is a * ones,
    so a spike scores 128 a / sqrt(128) * log2 e; the other keys score near 0."""
    Hq, Hkv, D, P = 16, 8, 128, 16
    prefix, extend = [272, 272, 400, 16], [24, 24, 24, 150]
    spikes = [{150: 1.875, 200: 2.0},  # block 1 at 32.6, a second spike 2 below it
              {150: 1.875, 200: 8.0},  # block 1 at 130.6
              {150: 1.0, 300: 4.0, 340: 3.875},  # block 1 at 16.3, block 2 at 65.3 (49 above it)
              {}]
    eb = _batch(prefix, extend, P, seed=3)
    pb = eb.paged
    rng = np.random.default_rng(8)
    N = pb.num_slots
    hk = O.round_to(rand(rng, (N, Hkv, D), "bfloat16") * np.float32(2.0 ** -6), "bfloat16")
    hv = rand(rng, (N, Hkv, D), "bfloat16")
    T = int(eb.extend.sum())
    q = np.ones((T, Hq, D), np.float32)
    q[T - extend[-1]:] = rand(rng, (extend[-1], Hq, D), "bfloat16")
    for b, sp in enumerate(spikes):
        for pos, a in sp.items():
            hk[pb.page_table[b, pos]] = np.float32(a)
    # the inputs make the jumps they are meant to (row 0 of each request, head 0)
    l2e = D ** -0.5 * np.log2(np.e)
    biggest = []
    for b in range(3):
        s2 = (hk[pb.page_table[b, : int(prefix[b]) + 1], 0] @ q[int(np.sum(extend[:b])), 0]) * l2e
        biggest.append(max(_max_jumps(s2)))
    assert 32 < biggest[0] < 33 and biggest[1] > 126 and 48 < biggest[2] < 50, biggest
    out, ref = _run_extend_arrays(eb, Hq, Hkv, D, "bfloat16", hk, hv, q)
    err = max_abs(out, ref)
    assert err <= TOL["bfloat16"], err


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_extend_config3_shapes(dtype):
    """Config 3 (32 ragged requests, prefix U[0,4096] page-aligned + one unaligned,
    extend U[64,512], 16/8/128, page 16), reduced to 8 requests for the fp64 oracle."""
    eb = W.config3_batch(seed=0, batch=8)
    out, ref = _run_extend(eb, 16, 8, 128, dtype, seed=4)
    err = max_abs(out, ref)
    assert err <= TOL[dtype], err


@pytest.mark.parametrize("P", [16, 1])
def test_extend_config3_full_benchmark_batch(P):
    """The whole config-3 batch the benchmark times (W.config3_batch(seed=0): 32 requests,
    ~9.1 k query rows, prefixes up to 4096; page 16 runs the tcgen05 kernel directly, page 1
    the page packer first). Oracle: the reference's prefill (attention/base.py:85-105) in
    float64 torch BLAS on the CPU, all rows compared."""
    import torch

    from minisgl_b200 import MHAKVCache
    from minisgl_b200.attention import B200AttnBackend

    eb = W.config3_batch(seed=0, page_size=P)
    pb = eb.paged
    assert pb.batch_size == 32
    Hq, Hkv, D = 16, 8, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    kv = MHAKVCache(1, pb.num_slots, Hkv, D, torch.bfloat16)
    kv.k[0].normal_(generator=gen)
    kv.v[0].normal_(generator=gen)
    T = int(eb.extend.sum())
    q = torch.randn((T, Hq, D), device="cuda", generator=gen).to(torch.bfloat16)
    be = B200AttnBackend(HeadConfig(Hq, Hkv, D), kv, pb.page_table, page_size=P)
    meta = be.extend_metadata_from_lens(pb.rows, pb.lens, eb.extend)
    assert (meta.pack is not None) == (P == 1) and meta.group_starts == (P == 1)
    out = be._forward_prefill(q, None, None, 0, meta).float().cpu()
    torch.cuda.synchronize()
    idx = [pb.page_table[b, : int(pb.lens[b])] for b in range(pb.batch_size)]
    qo = np.concatenate([[0], np.cumsum(eb.extend)])
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = O.forward_prefill_torch(q.cpu(), kv.k[0].cpu(), kv.v[0].cpu(), qo, idx, D ** -0.5)
    err = float((out.double() - ref).abs().max())
    assert err <= TOL["bfloat16"], err


@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8)])
def test_extend_page1_runs_read_in_place_fragments_packed(hq, hkv):
    """Page size 1, bf16 (b2a_extend_groups): 16-key groups that are one run of consecutive
    slots are read in place, the others are packed into the staging pool first. The
    requests mix the cases: one run from an unaligned slot, random slots, two runs that
    meet inside a group, a run that ends at the pool's last slot (its last group's box
    reaches past the pool), a fresh prompt, one query over a short run."""
    rng = np.random.default_rng(11)
    N = 6000
    prefix = np.array([200, 150, 24, 40, 0, 16], np.int64)
    extend = np.array([70, 33, 40, 5, 129, 1], np.int64)
    lens = prefix + extend
    free = rng.permutation(np.arange(2000, 5000))
    table = np.zeros((len(lens), int(lens.max())), np.int32)
    table[0, :270] = 37 + np.arange(270)
    table[1, :183] = free[:183]
    table[2, :64] = np.concatenate([400 + np.arange(24), 900 + np.arange(40)])
    table[3, :45] = N - 45 + np.arange(45)
    table[4, :129] = 1200 + np.arange(129)
    table[5, :17] = 1500 + np.arange(17)
    pb = W.PagedBatch(table, np.arange(len(lens)), lens, 1, N)
    eb = W.ExtendBatch(pb, prefix, extend)
    out, ref = _run_extend(eb, hq, hkv, 128, "bfloat16", seed=12)
    err = max_abs(out, ref)
    assert err <= TOL["bfloat16"], err


def test_extend_page1_group_metadata():
    """Which groups are read in place and where the packed ones start (host metadata)."""
    import torch

    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.kvcache import MHAKVCache

    N = 1000
    lens = np.array([40, 20, 16], np.int64)
    table = np.zeros((3, 40), np.int32)
    table[0, :40] = 37 + np.arange(40)
    table[1, :20] = [5, 9, 3, 700, 701, 702, 703, 704, 705, 706, 707, 708, 709, 710, 711, 712, 800, 801, 802, 803]
    table[2, :16] = np.concatenate([500 + np.arange(8), 600 + np.arange(8)])
    kv = MHAKVCache(1, N, 8, 128, torch.bfloat16)
    be = B200AttnBackend(HeadConfig(16, 8, 128), kv, table, page_size=1)
    meta = be.extend_metadata_from_lens(np.arange(3), lens, np.array([4, 4, 4]))
    assert meta.group_starts and meta.page_size == 16
    np.testing.assert_array_equal(to_np(meta.kv_indptr), [0, 3, 5, 6])
    # request 0: runs at 37, 53, 69 (the last of 8 keys); request 1: its first group is not a
    # run (staging page 0), its 4-key tail is (800); request 2: two runs of 8 (staging page 1)
    np.testing.assert_array_equal(to_np(meta.kv_indices), [37, 53, 69, N, 800, N + 16])
    np.testing.assert_array_equal(to_np(meta.kv_last_page_len), [8, 4, 16])
    pk = meta.pack
    assert pk.n_groups == 2 and pk.out_slots == 32
    np.testing.assert_array_equal(to_np(pk.src_kv_indices), np.concatenate([table[1, :16], table[2, :16]]))


def test_extend_single_request_long_prefix_bf16():
    eb = _batch([4000], [512], 16, seed=3)
    out, ref = _run_extend(eb, 16, 8, 128, "bfloat16", seed=5)
    assert max_abs(out, ref) <= TOL["bfloat16"]


@pytest.mark.parametrize("P", [1, 2, 8])
def test_pack_kv_rows_bit_exact(P):
    """b2a_pack_kv: every request's rows land at out_page_indptr[b] * 16 + p, byte for byte."""
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.attention.base import paged_kv_indices

    rng = np.random.default_rng(7)
    lens = np.array([1, 15, 16, 17, 200, 33])
    pb = W.allocate_pages(lens, 4096, P, rng)
    Hkv, D = 8, 128
    k_pool = torch.randn((4096, Hkv, D), device="cuda").to(torch.bfloat16)
    v_pool = torch.randn((4096, Hkv, D), device="cuda").to(torch.bfloat16)
    kv_indptr, kv_indices, _ = paged_kv_indices(pb.page_table, pb.rows, pb.lens, P)
    tok = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    npg = (lens + 15) // 16
    opi = np.concatenate([[0], np.cumsum(npg)]).astype(np.int32)
    out_slots = int(opi[-1]) * 16
    k_out = torch.zeros((out_slots, Hkv, D), dtype=torch.bfloat16, device="cuda")
    v_out = torch.zeros_like(k_out)
    dev = [torch.from_numpy(x).cuda() for x in (kv_indptr, kv_indices, tok, opi)]
    nat.call("b2a_pack_kv", k_pool.data_ptr(), v_pool.data_ptr(), 4096, dev[0].data_ptr(), dev[1].data_ptr(), P,
             dev[2].data_ptr(), dev[3].data_ptr(), len(lens), int(tok[-1]), Hkv, D, nat.B2A_DTYPE_BF16,
             k_out.data_ptr(), v_out.data_ptr(), out_slots, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    kp, vp, ko, vo = (t.view(torch.int16).cpu().numpy() for t in (k_pool, v_pool, k_out, v_out))
    for b, L in enumerate(lens.tolist()):
        src = pb.page_table[b, :L]
        dst = opi[b] * 16 + np.arange(L)
        assert np.array_equal(ko[dst], kp[src]) and np.array_equal(vo[dst], vp[src])
        tail = np.arange(opi[b] * 16 + L, opi[b + 1] * 16)
        assert not ko[tail].any() and not vo[tail].any()  # rows past the request stay untouched


def test_pack_kv_row_list_bit_exact():
    """b2a_pack_kv row-list form: staging row g = pool row kv_indices[g], byte for byte;
    a source outside the pool is skipped (row left as it was) and reported."""
    import torch

    from minisgl_b200 import _native as nat

    rng = np.random.default_rng(8)
    Hkv, D, N = 8, 128, 4096
    k_pool = torch.randn((N, Hkv, D), device="cuda").to(torch.bfloat16)
    v_pool = torch.randn((N, Hkv, D), device="cuda").to(torch.bfloat16)
    src = rng.integers(0, N, 48).astype(np.int32)
    src[20] = N + 3  # outside the pool
    k_out = torch.zeros((48, Hkv, D), dtype=torch.bfloat16, device="cuda")
    v_out = torch.zeros_like(k_out)
    s = torch.from_numpy(src).cuda()
    nat.call("b2a_pack_kv", k_pool.data_ptr(), v_pool.data_ptr(), N, None, s.data_ptr(), 1, None, None, 3, 48, Hkv,
             D, nat.B2A_DTYPE_BF16, k_out.data_ptr(), v_out.data_ptr(), 48, torch.cuda.current_stream().cuda_stream)
    code = nat.ctypes.c_int(0)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, nat.ctypes.byref(code))
    assert code.value == 32
    kp, vp, ko, vo = (t.view(torch.int16).cpu().numpy() for t in (k_pool, v_pool, k_out, v_out))
    ok = np.arange(48) != 20
    assert np.array_equal(ko[ok], kp[src[ok]]) and np.array_equal(vo[ok], vp[src[ok]])
    assert not ko[20].any() and not vo[20].any()
