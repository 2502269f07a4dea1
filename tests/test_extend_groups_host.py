"""Host logic of the small-page extend (b2a_extend_groups): which 16-key groups are read in place
and which are packed, checked against a direct per-group restatement on random slot layouts.

A group of 16 keys is read in place when its slots are one run of consecutive slots that lies
wholly inside the pool; every other group gets the next staging page, in group order, with its
source slots as 16 rows (a short last group repeats its last slot).
"""

from __future__ import annotations

import numpy as np
import pytest

from minisgl_b200.attention.b200 import extend_key_groups


def _direct(slot_lists, num_slots, Q=16):
    starts, rows, lpl, group_indptr = [], [], [], [0]
    for sl in slot_lists:
        L = len(sl)
        n = (L + Q - 1) // Q
        for j in range(n):
            g = sl[j * Q:(j + 1) * Q]
            run = all(g[i] == g[0] + i for i in range(len(g))) and g[0] >= 0 and g[0] + len(g) <= num_slots
            if run:
                starts.append(int(g[0]))
            else:
                starts.append(num_slots + len(rows))
                rows += [int(x) for x in g] + [int(g[-1])] * (Q - len(g))
        lpl.append(L - (n - 1) * Q if n else 0)
        group_indptr.append(group_indptr[-1] + n)
    return group_indptr, starts, lpl, rows


def _layout(rng, L, P, num_pages):
    """Page ids of one request: consecutive runs of random length at random starts, with the
    odd random page and, rarely, an id outside the pool."""
    n = (L + P - 1) // P
    out = []
    while len(out) < n:
        kind = rng.random()
        if kind < 0.6:
            run = int(rng.integers(1, 40))
            s = int(rng.integers(0, num_pages))
            out += list(range(s, s + run))
        elif kind < 0.95:
            out.append(int(rng.integers(0, num_pages)))
        else:
            out.append(num_pages + int(rng.integers(0, 5)))  # past the pool
    return np.array(out[:n], np.int64)


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_extend_key_groups_match_direct_restatement(P):
    rng = np.random.default_rng(P)
    num_pages = 3000 // P
    num_slots = num_pages * P
    for _ in range(40):
        B = int(rng.integers(1, 9))
        lens = rng.integers(0, 300, B)
        pages = [_layout(rng, int(L), P, num_pages) for L in lens]
        indptr = np.zeros(B + 1, np.int64)
        np.cumsum([len(p) for p in pages], out=indptr[1:])
        indices = np.concatenate(pages) if B else np.zeros(0, np.int64)
        slot_lists = [np.concatenate([np.arange(p * P, p * P + P) for p in pg])[:L] if L else np.zeros(0, np.int64)
                      for pg, L in zip(pages, lens)]
        gi, st, lp, rows = extend_key_groups(lens, indptr, indices, P, num_slots)
        w_gi, w_st, w_lp, w_rows = _direct(slot_lists, num_slots)
        np.testing.assert_array_equal(gi, w_gi)
        np.testing.assert_array_equal(st, w_st)
        np.testing.assert_array_equal(lp, w_lp)
        np.testing.assert_array_equal(rows, np.array(w_rows, np.int64).reshape(-1))


def test_extend_key_groups_fresh_allocator_needs_no_staging():
    """A fresh free list hands every prompt one run: with 16-aligned request boundaries in key
    space every group is read in place, whatever the run's first slot."""
    lens = np.array([16, 100, 33, 1])
    starts0 = np.array([5, 21, 121, 154])
    slots = np.concatenate([np.arange(s, s + L) for s, L in zip(starts0, lens)])
    indptr = np.concatenate([[0], np.cumsum(lens)])
    gi, st, lp, rows = extend_key_groups(lens, indptr, slots, 1, 200)
    assert len(rows) == 0
    np.testing.assert_array_equal(st, [5, 21, 37, 53, 69, 85, 101, 117, 121, 137, 153, 154])
    np.testing.assert_array_equal(lp, [16, 4, 1, 1])
