"""Host logic of the engine harness: radix prefix cache and request managers (CPU).

Cases follow the reference's behaviour (kvcache/radix_cache.py, scheduler/
cache.py, scheduler/prefill.py): page-aligned matching with node splits,
reference counts that protect matched prefixes, LRU eviction of unreferenced
leaves, ownership hand-over of a request's KV to the prefix cache, chunked
prefill under the token budget and conservative KV admission.
"""

from __future__ import annotations

import numpy as np
import pytest

from minisgl_b200.core import Batch, Req, SamplingParams
from minisgl_b200.engine.managers import CacheManager, ChunkedReq, DecodeManager, PrefillManager, TableManager
from minisgl_b200.engine.radix import NaivePrefixCache, RadixPrefixCache


def ids(*xs):
    return np.array(xs, dtype=np.int32)


@pytest.mark.parametrize("P", [1, 4])
def test_radix_insert_match_split(P):
    rc = RadixPrefixCache(P)
    a = np.arange(1, 13, dtype=np.int32)  # 12 tokens
    slots = np.arange(100, 112, dtype=np.int32)
    dup, h = rc.insert_prefix(a, slots)
    assert dup == 0 and h.cached_len == 12 and rc.size_info == (12, 0)
    # shares the first 6 tokens: a page-aligned match of 6 (P=1) or 4 (P=4), splitting the node
    b = np.concatenate([a[:6], ids(99, 98, 97, 96, 95, 94)])
    m = rc.match_prefix(b).handle
    want = 6 if P == 1 else 4
    assert m.cached_len == want
    assert np.array_equal(m.get_matched_indices(), slots[:want])
    rc.check_integrity()
    # inserting b adds only its new suffix
    dup, hb = rc.insert_prefix(b, np.arange(200, 212, dtype=np.int32))
    assert dup == want and hb.cached_len == 12
    assert rc.size_info.total_size == 12 + (12 - want)
    rc.check_integrity()


def test_radix_partial_page_not_matched():
    rc = RadixPrefixCache(4)
    rc.insert_prefix(np.arange(10, dtype=np.int32), np.arange(10, dtype=np.int32))  # 8 tokens kept (2 pages)
    assert rc.size_info.total_size == 8
    assert rc.match_prefix(np.arange(3, dtype=np.int32)).handle.cached_len == 0  # under one page
    assert rc.match_prefix(np.arange(7, dtype=np.int32)).handle.cached_len == 4


def test_radix_lock_and_lru_eviction():
    rc = RadixPrefixCache(1)
    _, ha = rc.insert_prefix(ids(1, 2, 3), ids(10, 11, 12))
    _, hb = rc.insert_prefix(ids(5, 6), ids(20, 21))
    rc.match_prefix(ids(1, 2, 3))  # a was used last: b is the LRU leaf
    rc.lock_handle(ha)
    assert rc.size_info == (2, 3)
    with pytest.raises(RuntimeError):
        rc.evict(3)  # only b is evictable
    assert sorted(rc.evict(2).tolist()) == [20, 21]
    rc.lock_handle(ha, unlock=True)
    assert rc.size_info == (3, 0)
    assert sorted(rc.evict(1).tolist()) == [10, 11, 12]  # a whole leaf goes
    assert rc.size_info == (0, 0)
    rc.check_integrity()


def test_radix_duplicate_insert_keeps_cached_slots_and_split_keeps_refs():
    rc = RadixPrefixCache(1)
    _, h = rc.insert_prefix(ids(1, 2, 3, 4), ids(10, 11, 12, 13))
    # a second request computed the same 4 tokens plus 2 more: its first 4 slots are
    # redundant (the caller frees them) and the tree keeps the slots it already had
    dup, h2 = rc.insert_prefix(ids(1, 2, 3, 4, 5, 6), ids(30, 31, 32, 33, 34, 35))
    assert dup == 4 and h2.cached_len == 6
    assert h2.get_matched_indices().tolist() == [10, 11, 12, 13, 34, 35]
    assert rc.size_info == (6, 0)
    # a lock taken before a split still covers both halves of the split node
    rc.lock_handle(h)
    assert rc.size_info == (2, 4)
    assert rc.match_prefix(ids(1, 2, 9)).handle.cached_len == 2  # splits [1,2,3,4] at 2
    rc.check_integrity()
    assert rc.size_info == (2, 4)
    rc.lock_handle(h, unlock=True)
    assert rc.size_info == (6, 0)
    rc.check_integrity()


def test_radix_evict_prefers_older_and_frees_parents():
    rc = RadixPrefixCache(1)
    rc.insert_prefix(ids(1, 2, 3, 4), ids(1, 2, 3, 4))
    rc.insert_prefix(ids(1, 2, 7, 8), ids(1, 2, 7, 8))  # splits: [1,2] -> [3,4], [7,8]
    rc.match_prefix(ids(1, 2, 7, 8))  # touch the [7,8] branch
    assert sorted(rc.evict(2).tolist()) == [3, 4]
    out = rc.evict(4)  # [7,8] then its parent [1,2], which became an unreferenced leaf
    assert sorted(out.tolist()) == [1, 2, 7, 8]
    assert rc.size_info == (0, 0)


def test_naive_cache():
    nc = NaivePrefixCache(16)
    assert nc.match_prefix(np.arange(40, dtype=np.int32)).handle.cached_len == 0
    assert nc.insert_prefix(np.arange(40, dtype=np.int32), np.arange(40, dtype=np.int32)).cached_len == 0
    with pytest.raises(RuntimeError):
        nc.evict(1)


def _mgrs(num_pages=64, P=4, rows=4, max_len=256, kind="radix"):
    pt = np.zeros((rows, max_len), dtype=np.int32)
    cache = CacheManager(num_pages, P, pt, kind)
    table = TableManager(rows, pt, device="cpu")
    dec = DecodeManager(P)
    return pt, cache, table, dec, PrefillManager(cache, table, dec)


def _finish_step(batch: Batch, cache: CacheManager, dec: DecodeManager, table: TableManager, token: int):
    """What the scheduler does after a step: complete, append, finish or cache the prompt."""
    for r in batch.reqs:
        r.complete_one()
    dec.filter_reqs(batch.reqs)
    with cache.lazy_free_region():
        for r in batch.reqs:
            if isinstance(r, ChunkedReq):
                continue
            r.append_host(token)
            if len(r.input_ids) >= r.max_device_len:
                dec.remove_req(r)
                table.free(r.table_idx)
                cache.cache_req(r, finished=True)
            elif batch.is_prefill:
                cache.cache_req(r, finished=False)


@pytest.mark.parametrize("P", [1, 4])
@pytest.mark.parametrize("kind", ["radix", "naive"])
def test_scheduling_loop_accounts_every_page(P, kind):
    """Chunked prefill + decode + prefix reuse on the host; at the end every page is free or cached."""
    pt, cache, table, dec, pre = _mgrs(num_pages=256 // P * 4, P=P, kind=kind)
    rng = np.random.default_rng(0)
    shared = rng.integers(0, 50, 40).astype(np.int32)
    prompts = [shared, np.concatenate([shared, rng.integers(0, 50, 10).astype(np.int32)]),
               rng.integers(0, 50, 70).astype(np.int32), shared[:25]]
    for uid, p in enumerate(prompts):
        pre.add_one_req(uid, p, SamplingParams(max_tokens=5, ignore_eos=True))
    steps, hits = 0, 0
    while pre.runnable or dec.runnable:
        batch = pre.schedule_next_batch(32) or dec.schedule_next_batch()
        assert batch is not None
        if batch.is_prefill:
            assert sum(r.extend_len for r in batch.reqs) <= 32  # the token budget holds
            hits += sum(r.cached_len for r in batch.reqs if r.cache_handle.cached_len == r.cached_len)
        cache.allocate_paged(batch.reqs)
        for r in batch.reqs:  # every token being computed has a slot inside the pool
            s = pt[r.table_idx, r.cached_len: r.device_len]
            assert s.min() >= 0 and s.max() < cache.num_pages * P
        _finish_step(batch, cache, dec, table, token=7)
        steps += 1
        assert steps < 200
    cache.check_integrity()
    assert table.available_size == 4
    if kind == "radix":
        assert hits > 0  # later prompts reused cached prefixes
        assert cache.prefix_cache.size_info.protected_size == 0
    else:
        assert len(cache.free_slots) == cache.num_pages


def test_admission_reserves_worst_case_kv():
    # 8 pages of 4 = 32 tokens: a 10-token prompt with max_tokens 20 needs 30, a second one does not fit
    pt, cache, table, dec, pre = _mgrs(num_pages=8, P=4)
    pre.add_one_req(0, np.arange(10, dtype=np.int32), SamplingParams(max_tokens=20))
    pre.add_one_req(1, np.arange(10, 20, dtype=np.int32), SamplingParams(max_tokens=20))
    b = pre.schedule_next_batch(4096)
    assert [r.uid for r in b.reqs] == [0]
    cache.allocate_paged(b.reqs)
    for r in b.reqs:
        r.complete_one()
    dec.filter_reqs(b.reqs)
    assert pre.schedule_next_batch(4096) is None  # still does not fit next to request 0's reservation


def test_chunked_prefill_continues_first():
    pt, cache, table, dec, pre = _mgrs(num_pages=64, P=4)
    pre.add_one_req(0, np.arange(50, dtype=np.int32), SamplingParams(max_tokens=2))
    pre.add_one_req(1, np.arange(60, 65, dtype=np.int32), SamplingParams(max_tokens=2))
    b1 = pre.schedule_next_batch(32)
    assert [type(r).__name__ for r in b1.reqs] == ["ChunkedReq"] and b1.reqs[0].extend_len == 32
    cache.allocate_paged(b1.reqs)
    for r in b1.reqs:
        r.complete_one()
    b2 = pre.schedule_next_batch(32)
    assert [r.uid for r in b2.reqs] == [0, 1]  # the chunked request continues ahead of the queue
    assert b2.reqs[0].cached_len == 32 and b2.reqs[0].extend_len == 18
    assert not isinstance(b2.reqs[0], ChunkedReq)


def test_router_keeps_prefix_groups_and_balances():
    from minisgl_b200.engine.router import route_requests

    rng = np.random.default_rng(3)
    sys_prompts = [rng.integers(0, 1000, 64).astype(np.int32) for _ in range(6)]
    prompts, owner = [], []
    for i in range(120):
        g = i % 6
        prompts.append(np.concatenate([sys_prompts[g], rng.integers(0, 1000, int(rng.integers(5, 200)))]))
        owner.append(g)
    for i in range(40):  # unrelated prompts
        prompts.append(rng.integers(1000, 2000, int(rng.integers(20, 300))).astype(np.int32))
        owner.append(-1)
    costs = np.array([len(p) for p in prompts]) + 100
    ranks = route_requests(prompts, costs, 4, page_size=16)
    assert sorted(np.concatenate(ranks).tolist()) == list(range(len(prompts)))
    rank_of = {int(i): r for r, ids in enumerate(ranks) for i in ids}
    for g in range(6):  # every shared-prefix group sits on one rank
        assert len({rank_of[i] for i in range(len(prompts)) if owner[i] == g}) == 1
    load = np.array([costs[ids].sum() for ids in ranks])
    assert load.max() <= 1.25 * load.mean()


def test_router_splits_an_oversized_group():
    from minisgl_b200.engine.router import route_requests

    common = np.arange(32, dtype=np.int32)
    prompts = [np.concatenate([common, [i]]).astype(np.int32) for i in range(64)]
    costs = np.full(64, 10.0)
    ranks = route_requests(prompts, costs, 4, page_size=16)
    load = np.array([costs[ids].sum() for ids in ranks])
    assert load.min() > 0 and load.max() <= 1.1 * load.mean()  # one giant group is still balanced
    assert route_requests(prompts, costs, 1, 16)[0].tolist() == list(range(64))


def _prompt(cm: CacheManager, tokens, row: int) -> Req:
    """Admit a prompt the way the prefill manager does: match, lock, borrow the slots."""
    toks = np.array(tokens, dtype=np.int32)
    h = cm.match_req(toks)
    cm.lock(h)
    cm.page_table[row, : h.cached_len] = h.get_matched_indices()
    return Req(input_ids=toks, table_idx=row, cached_len=h.cached_len, output_len=4, cache_handle=h)


def _prefill_and_finish(cm: CacheManager, tokens, row: int = 0) -> Req:
    r = _prompt(cm, tokens, row)
    cm.allocate_paged([r])
    r.complete_one()
    cm.cache_req(r, finished=True)
    return r


def test_cache_manager_reuse_recomputes_the_last_prompt_token():
    pt = np.zeros((4, 64), dtype=np.int32)
    cm = CacheManager(32, 1, pt, "radix")
    _prefill_and_finish(cm, [1, 2, 3, 4, 5])
    assert cm.prefix_cache.size_info.evictable_size == 5
    cm.check_integrity()
    # the same prompt again: its last token is computed anyway (its logits pick the
    # next token), so only 4 of the 5 cached tokens are reused
    same = _prompt(cm, [1, 2, 3, 4, 5], row=2)
    assert same.cached_len == 4
    cm.unlock(same.cache_handle)
    # a longer prompt that starts with the whole cached one reuses all 5
    longer = _prompt(cm, [1, 2, 3, 4, 5, 6, 7], row=1)
    assert longer.cached_len == 5
    cm.allocate_paged([longer])
    longer.complete_one()
    cm.cache_req(longer, finished=True)
    cm.check_integrity()
    assert cm.prefix_cache.size_info == (7, 0)


def test_cache_manager_evicts_cached_prefixes_when_full():
    pt = np.zeros((4, 64), dtype=np.int32)
    cm = CacheManager(8, 1, pt, "radix")
    _prefill_and_finish(cm, [1, 2, 3, 4, 5, 6])
    assert len(cm.free_slots) == 2 and cm.available_size == 8
    _prefill_and_finish(cm, [9, 9, 9, 9, 9], row=1)  # needs 5 slots: evicts the old prefix
    cm.check_integrity()
    assert cm.prefix_cache.size_info.total_size == 5


def test_cache_manager_pages_of_four():
    pt = np.zeros((4, 64), dtype=np.int32)
    cm = CacheManager(8, 4, pt, "radix")
    r = _prefill_and_finish(cm, list(range(10)))  # 10 tokens take 3 pages
    pages = pt[r.table_idx, :12].reshape(3, 4)
    assert np.all(pages[:, 0] % 4 == 0) and np.all(pages - pages[:, :1] == np.arange(4))
    # the 2 full pages go to the prefix cache, the partial third page back to the free list
    assert cm.prefix_cache.size_info.evictable_size == 8 and len(cm.free_slots) == 6
    assert np.all(cm.free_slots % 4 == 0)
    cm.check_integrity()
