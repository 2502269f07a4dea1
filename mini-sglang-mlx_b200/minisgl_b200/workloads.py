"""Seeded synthetic batches with the shapes of the benchmark configurations.

There is no public dataset for this path; these generators stand in for the
reference's random-token workloads (benchmark/offline.py:19-23,
tutorials/ch04_attention.py:19-43) with explicit seeds. They build the host
structures the scheduler would produce -- a token-granular page table whose
pages are P-aligned runs of P slots taken from a shuffled free list
(scheduler/cache.py:28-72) -- plus per-request lengths. Tensor contents are
drawn separately (numpy for CPU-sized cases, torch on the device for pools of
tens of GB).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np


@dataclass
class PagedBatch:
    page_table: np.ndarray  # int32 [B, max_seq_len] token -> slot
    rows: np.ndarray  # int64 [B] page-table row of each request
    lens: np.ndarray  # int64 [B] tokens in the KV cache (decode) or device_len (extend)
    page_size: int
    num_slots: int

    @property
    def batch_size(self) -> int:
        return int(self.lens.shape[0])


def allocate_pages(lens: np.ndarray, num_slots: int, page_size: int, rng: np.random.Generator,
                   max_seq_len: int | None = None) -> PagedBatch:
    """Give each request ceil(len / P) pages from a shuffled free list (fragmented pool)."""
    lens = np.asarray(lens, dtype=np.int64)
    P = page_size
    num_pages = num_slots // P
    need = (lens + P - 1) // P
    if int(need.sum()) > num_pages:
        raise ValueError(f"pool of {num_slots} slots cannot hold {int(lens.sum())} tokens")
    free = rng.permutation(num_pages).astype(np.int64)
    max_seq_len = max_seq_len or int(need.max(initial=1)) * P
    table = np.zeros((len(lens), max_seq_len), dtype=np.int32)
    ar = np.arange(P, dtype=np.int64)
    off = 0
    for b, n in enumerate(need.tolist()):  # request b takes the next n pages of the shuffled list
        m = min(n * P, max_seq_len)
        table[b, :m] = (free[off:off + n, None] * P + ar[None, :]).reshape(-1)[:m]
        off += n
    return PagedBatch(table, np.arange(len(lens), dtype=np.int64), lens, P, num_slots)


def permutation_slots(lens: np.ndarray, num_slots: int, rng: np.random.Generator) -> PagedBatch:
    """page_size 1: each request's tokens on disjoint slots of one seeded permutation
    (tests/test_attention.py:22-32 layout)."""
    lens = np.asarray(lens, dtype=np.int64)
    perm = rng.permutation(num_slots).astype(np.int32)
    table = np.zeros((len(lens), int(lens.max(initial=1))), dtype=np.int32)
    off = 0
    for b, n in enumerate(lens.tolist()):
        table[b, :n] = perm[off:off + n]
        off += n
    return PagedBatch(table, np.arange(len(lens), dtype=np.int64), lens, 1, num_slots)


# ---------------------------------------------------------------- configurations
CONFIG1 = dict(B=8, Hq=16, Hkv=8, D=128, dtype="float32", page_size=1, num_slots=16384, lo=100, hi=1024)
CONFIG2 = dict(B=128, Hq=16, Hkv=8, D=128, dtype="bfloat16", page_size=16, num_slots=262144, lo=100,
               hi=2048, layers=28)
CONFIG3 = dict(B=32, Hq=16, Hkv=8, D=128, dtype="bfloat16", page_size=16, prefix_hi=4096, ext_lo=64,
               ext_hi=512, theta=1e6)
CONFIG5 = dict(B=1024, Hq=32, Hkv=8, D=128, dtype="bfloat16", page_size=16, lo=1024, hi=131072, layers=36)
CONFIG4 = dict(num_seqs=256, max_input=1024, max_output=1024, vocab_hi=10000, max_running_req=128,
               max_extend_tokens=4096, num_tokens=131072, page_size=16)


def config1_batch(seed: int = 0) -> PagedBatch:
    c = CONFIG1
    rng = np.random.default_rng(seed)
    lens = rng.integers(c["lo"], c["hi"] + 1, size=c["B"])
    return permutation_slots(lens, c["num_slots"], rng)


def config2_batch(seed: int = 0, batch: int | None = None) -> PagedBatch:
    c = CONFIG2
    rng = np.random.default_rng(seed)
    lens = rng.integers(c["lo"], c["hi"] + 1, size=batch or c["B"])
    return allocate_pages(lens, c["num_slots"], c["page_size"], rng)


@dataclass
class ExtendBatch:
    paged: PagedBatch  # lens = prefix + extend (device_len)
    prefix: np.ndarray  # cached_len
    extend: np.ndarray  # extend_len


def config3_batch(seed: int = 0, batch: int | None = None, num_slots: int | None = None,
                  page_size: int | None = None) -> ExtendBatch:
    """32 requests, prefix U[0,4096] aligned down to the page size (radix matches are page
    aligned, kvcache/radix_cache.py:254) except request 0 which keeps an unaligned prefix;
    extend U[64,512]."""
    c = CONFIG3
    P = page_size or c["page_size"]
    rng = np.random.default_rng(seed)
    B = batch or c["B"]
    prefix = rng.integers(0, c["prefix_hi"] + 1, size=B)
    unaligned = prefix[0]
    prefix = prefix // P * P
    prefix[0] = unaligned
    extend = rng.integers(c["ext_lo"], c["ext_hi"] + 1, size=B)
    lens = prefix + extend
    slots = num_slots or int(((lens + P - 1) // P * P).sum() * 2 + 1024) // P * P
    paged = allocate_pages(lens, slots, P, rng)
    return ExtendBatch(paged, prefix.astype(np.int64), extend.astype(np.int64))


def config5_lens(seed: int = 0, batch: int | None = None) -> np.ndarray:
    """Context lengths log-uniform in [1024, 131072]."""
    c = CONFIG5
    rng = np.random.default_rng(seed)
    u = rng.uniform(np.log(c["lo"]), np.log(c["hi"]), size=batch or c["B"])
    return np.floor(np.exp(u)).astype(np.int64)


def config4_workload(seed: int = 0, num_seqs: int | None = None):
    """Offline e2e workload (benchmark/offline.py:19-23 shapes): prompts of U[100, 1024] random
    token ids in [0, 10000], output lengths U[100, 1024]. Returns (prompts, out_lens)."""
    c = CONFIG4
    rng = np.random.default_rng(seed)
    n = num_seqs or c["num_seqs"]
    prompts = [rng.integers(0, c["vocab_hi"] + 1, int(rng.integers(100, c["max_input"] + 1))).astype(np.int32)
               for _ in range(n)]
    out_lens = rng.integers(100, c["max_output"] + 1, n).astype(np.int64)
    return prompts, out_lens


CONFIG4_SHARED = dict(num_groups=16, per_group=16, sys_lo=512, sys_hi=2048, user_lo=100, user_hi=1024,
                      max_output=1024, vocab_hi=10000, max_running_req=128, max_extend_tokens=4096,
                      num_tokens=262144, page_size=16)


def config4_shared_workload(seed: int = 0):
    """Config 4 with shared prefixes: 16 system prompts of U[512, 2048] random token ids,
    each the start of 16 requests whose own part is U[100, 1024] tokens; outputs
    U[100, 1024]; the 256 requests arrive in a seeded random order. This is the traffic
    the prefix cache (kvcache/radix_cache.py) and the prefix-affinity router exist for.
    Returns (prompts, out_lens, group id of each request)."""
    c = CONFIG4_SHARED
    rng = np.random.default_rng(seed)
    systems = [rng.integers(0, c["vocab_hi"] + 1, int(rng.integers(c["sys_lo"], c["sys_hi"] + 1))).astype(np.int32)
               for _ in range(c["num_groups"])]
    n = c["num_groups"] * c["per_group"]
    group = np.repeat(np.arange(c["num_groups"]), c["per_group"])[rng.permutation(n)]
    prompts = [np.concatenate([systems[g], rng.integers(0, c["vocab_hi"] + 1,
                                                        int(rng.integers(c["user_lo"], c["user_hi"] + 1)))]).astype(np.int32)
               for g in group.tolist()]
    out_lens = rng.integers(100, c["max_output"] + 1, n).astype(np.int64)
    return prompts, out_lens, group


def shard_requests(costs: np.ndarray, world: int) -> List[np.ndarray]:
    """Longest-processing-time assignment of requests to `world` ranks.

    Requests are independent (no cross-request reduction in attention), so the
    batch is partitioned, never communicated. Returns the request ids of each
    rank, each sorted ascending.
    """
    costs = np.asarray(costs, dtype=np.float64)
    order = np.argsort(-costs, kind="stable")
    load = np.zeros(world)
    shards: List[list] = [[] for _ in range(world)]
    for i in order.tolist():
        r = int(np.argmin(load))
        shards[r].append(i)
        load[r] += costs[i]
    return [np.array(sorted(s), dtype=np.int64) for s in shards]
