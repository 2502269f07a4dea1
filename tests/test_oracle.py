"""CPU checks of the oracle itself: known answers and the reference's own invariants.

The reference ships no golden vectors (its decode test draws unseeded MLX
normals, tests/test_attention.py:24-26), so the oracle is pinned here by
hand-computable cases, by closed forms, and by the identities the reference
relies on (naive == per-request contiguous SDPA, attention/naive.py vs
tests/test_attention.py:10-16).
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import attention as O


def test_bf16_round_matches_torch():
    import torch

    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, 1.0, 1.00390625, 1.005859375, 3.4e38, -1e-40], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    np.testing.assert_array_equal(O.bf16_round(x), ref)


def test_single_key_returns_value():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 4, 1, 16))
    k = rng.standard_normal((1, 2, 1, 16))
    v = rng.standard_normal((1, 2, 1, 16))
    o = O.sdpa(q, k, v, 0.25)
    np.testing.assert_allclose(o[0, :2, 0], np.repeat(v[0, :1, 0], 2, 0), rtol=0, atol=1e-15)
    np.testing.assert_allclose(o[0, 2:, 0], np.repeat(v[0, 1:, 0], 2, 0), rtol=0, atol=1e-15)


def test_identical_keys_give_mean_of_values():
    rng = np.random.default_rng(3)
    k = np.repeat(rng.standard_normal((1, 1, 1, 8)), 5, axis=2)
    v = rng.standard_normal((1, 1, 5, 8))
    q = rng.standard_normal((1, 1, 1, 8))
    np.testing.assert_allclose(O.sdpa(q, k, v, 1.0)[0, 0, 0], v[0, 0].mean(0), atol=1e-14)


def test_one_hot_query_selects_key():
    D, L = 16, 9
    k = np.eye(L, D)[None, None] * 50.0
    v = np.arange(L * D, dtype=np.float64).reshape(1, 1, L, D)
    q = np.zeros((1, 1, 1, D))
    q[..., 4] = 1.0
    o = O.sdpa(q, k, v, 1.0)
    np.testing.assert_allclose(o[0, 0, 0], v[0, 0, 4], atol=1e-12)


def test_causal_is_bottom_right_aligned():
    rng = np.random.default_rng(4)
    Lq, Lkv, D = 3, 7, 8
    q = rng.standard_normal((1, 1, Lq, D))
    k = rng.standard_normal((1, 1, Lkv, D))
    v = rng.standard_normal((1, 1, Lkv, D))
    o = O.sdpa(q, k, v, 0.5, causal=True)
    for i in range(Lq):
        visible = Lkv - Lq + i + 1
        ref = O.sdpa(q[:, :, i:i + 1], k[:, :, :visible], v[:, :, :visible], 0.5)
        np.testing.assert_allclose(o[:, :, i:i + 1], ref, atol=1e-14)


@pytest.mark.parametrize("hq,hkv,d", [(16, 8, 128), (32, 8, 128), (8, 8, 64), (16, 2, 256)])
def test_naive_decode_equals_per_request_reference(hq, hkv, d):
    """The reference test's case list (tests/test_attention.py:19-32) on the oracle:
    naive padded gather + mask equals per-request contiguous SDPA."""
    rng = np.random.default_rng(0)
    N, B = 4096, 7
    lens = [1, 2, 17, 31, 32, 33, 700]
    k_pool = rng.standard_normal((N, hkv, d)).astype(np.float32)
    v_pool = rng.standard_normal((N, hkv, d)).astype(np.float32)
    q = rng.standard_normal((B, hq, d)).astype(np.float32)
    perm = rng.permutation(N).astype(np.int32)
    per_req, off = [], 0
    table = np.zeros((B, 1024), np.int32)
    for b, n in enumerate(lens):
        per_req.append(perm[off:off + n])
        table[b, :n] = per_req[-1]
        off += n
    idx, mask = O.naive_prepare_decode(table, np.arange(B), lens)
    assert idx.shape[1] == 768  # align_up(700, 128)
    out = O.naive_forward_decode(q, k_pool, v_pool, idx, mask, d ** -0.5)
    ref = O.reference_decode_per_request(q, k_pool, v_pool, per_req, d ** -0.5)
    np.testing.assert_allclose(out, ref, atol=1e-12)
    indptr, flat = O.metal_prepare_decode(table, np.arange(B), lens)
    np.testing.assert_array_equal(indptr, np.concatenate([[0], np.cumsum(lens)]))
    np.testing.assert_array_equal(flat, np.concatenate(per_req))


def test_rope_position_zero_is_identity():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((4, 3, 128)).astype(np.float32)
    inv = O.rope_inv_freq(128, 1e6)
    y = O.rope(x, np.zeros(4, np.int32), 128, inv)
    np.testing.assert_array_equal(y, x)


def test_rope_closed_form():
    """Rotate-half rule for one pair, against a hand-written rotation in float64."""
    D, base, p = 8, 10000.0, 37
    x = np.arange(1, D + 1, dtype=np.float32)[None, None]
    inv = O.rope_inv_freq(D, base)
    y = O.rope(x, np.array([p], np.int32), D, inv)[0, 0]
    for i in range(D // 2):
        ang = float(np.float32(np.float32(p) * inv[i]))
        c, s = math.cos(ang), math.sin(ang)
        x1, x2 = float(x[0, 0, i]), float(x[0, 0, i + D // 2])
        assert abs(y[i] - np.float32(x1 * c - x2 * s)) <= 1e-6
        assert abs(y[i + D // 2] - np.float32(x2 * c + x1 * s)) <= 1e-6
    # inverse frequencies: base^(-2i/D)
    np.testing.assert_allclose(inv, [base ** (-2 * i / D) for i in range(D // 2)], rtol=1e-7)


def test_rope_partial_rotary_passes_tail_through():
    rng = np.random.default_rng(6)
    x = rng.standard_normal((5, 2, 128)).astype(np.float32)
    inv = O.rope_inv_freq(64, 1e4)
    y = O.rope(x, np.arange(5, dtype=np.int32) * 1000, 64, inv)
    np.testing.assert_array_equal(y[..., 64:], x[..., 64:])
    assert not np.allclose(y[1:, :, :64], x[1:, :, :64])


def test_prefill_no_prefix_uses_fresh_kv_and_prefix_uses_pool():
    """attention/base.py:90-96: both branches must agree when the pool holds the fresh rows."""
    rng = np.random.default_rng(7)
    Hq, Hkv, D, N = 4, 2, 32, 256
    k_pool = rng.standard_normal((N, Hkv, D))
    v_pool = rng.standard_normal((N, Hkv, D))
    table = rng.permutation(N).astype(np.int32)[None, :100]
    q = rng.standard_normal((10, Hq, D))
    k = k_pool[table[0, 90:100]]
    v = v_pool[table[0, 90:100]]
    # cached_len 90 -> pool branch; the same 10 rows as "fresh" with cached_len 0 over a 10-token table
    meta = O.prepare_prefill(table, [0], [90], [100])
    o1 = O.forward_prefill(q, k, v, k_pool, v_pool, meta, D ** -0.5)
    assert meta.kv_indices[0] is not None and meta.last_indices.tolist() == [9]
    sub = table[:, 90:100]
    meta0 = O.prepare_prefill(sub, [0], [0], [10])
    o0 = O.forward_prefill(q, k, v, k_pool, v_pool, meta0, D ** -0.5)
    assert meta0.kv_indices[0] is None
    # o0 attends the 10 fresh rows only (causal); o1 attends the 90 cached rows too
    assert o0.shape == o1.shape == (10, Hq, D)
    kk = k_pool[table[0]].transpose(1, 0, 2)[None]
    vv = v_pool[table[0]].transpose(1, 0, 2)[None]
    ref_last = O.sdpa(q[-1][None, :, None, :], kk, vv, D ** -0.5)  # last row sees all 100 keys
    np.testing.assert_allclose(o1[-1], ref_last[0, :, 0], atol=1e-12)
    ref_first = O.sdpa(q[0][None, :, None, :], kk[:, :, :91], vv[:, :, :91], D ** -0.5)
    np.testing.assert_allclose(o1[0], ref_first[0, :, 0], atol=1e-12)
    ref0 = O.sdpa(q[3][None, :, None, :], kk[:, :, 90:94], vv[:, :, 90:94], D ** -0.5)
    np.testing.assert_allclose(o0[3], ref0[0, :, 0], atol=1e-12)


def test_torch_prefill_restatement_matches_numpy_oracle():
    """forward_prefill_torch (BLAS, for benchmark-sized parity tests) computes what
    forward_prefill computes: ragged requests, with and without prefix, Lq = 1 unmasked."""
    import torch

    rng = np.random.default_rng(11)
    prefix = np.array([0, 5, 33, 100, 0])
    ext = np.array([1, 17, 64, 3, 9])
    lens = prefix + ext
    N, Hq, Hkv, D = 1024, 16, 8, 64
    k, v = rng.standard_normal((N, Hkv, D)), rng.standard_normal((N, Hkv, D))
    q = rng.standard_normal((int(ext.sum()), Hq, D))
    table = np.stack([rng.permutation(N)[: lens.max()] for _ in lens]).astype(np.int32)
    meta = O.prepare_prefill(table, np.arange(len(lens)), prefix, lens)
    idx = [table[r, :n] for r, n in enumerate(lens)]
    meta.kv_indices = idx
    a = O.forward_prefill(q, None, None, k, v, meta, D ** -0.5)
    b = O.forward_prefill_torch(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), meta.q_offsets, idx,
                                D ** -0.5).numpy()
    assert np.abs(a - b).max() < 1e-12
