"""Host-side request managers of the engine harness.

Behaviour follows the reference scheduler package:
* ``CacheManager``  scheduler/cache.py:27-143   KV slots by page + prefix cache
* ``TableManager``  scheduler/table.py:7-34     page-table rows + last-token pool
* ``PrefillManager`` scheduler/prefill.py:42-141 FCFS admission, chunked prefill
* ``DecodeManager`` scheduler/decode.py:9-44    the running set

A KV page is free, owned by one request (its page-table row), or owned by the
prefix cache (shared while referenced, evictable otherwise). Admission is
conservative exactly as in the reference: a request is admitted only if its
remaining prompt plus its full ``max_tokens`` fit next to what the running
requests may still need, so a running request never runs out of KV.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import List, Set, Tuple

import numpy as np
import torch

from ..core import Batch, Req
from .radix import PrefixHandle, create_prefix_cache


def _ceil_div(a: int, b: int) -> int:
    return -(-a // b)


class CacheManager:
    def __init__(self, num_pages: int, page_size: int, page_table: np.ndarray, cache_type: str = "radix") -> None:
        self.page_size = page_size
        self.num_pages = num_pages
        self.page_table = page_table
        # free pages, each stored as the first slot of the page
        self.free_slots = np.arange(num_pages, dtype=np.int32) * page_size
        self.prefix_cache = create_prefix_cache(cache_type, page_size)
        self._pending_free: List[np.ndarray] | None = None

    # ------------------------------------------------------------ prefix cache
    def match_req(self, input_ids: np.ndarray) -> PrefixHandle:
        """Longest cached prefix of the prompt without its last token (which must be computed)."""
        assert len(input_ids) > 0
        return self.prefix_cache.match_prefix(input_ids[: len(input_ids) - 1]).handle

    def lock(self, handle: PrefixHandle) -> None:
        self.prefix_cache.lock_handle(handle, unlock=False)

    def unlock(self, handle: PrefixHandle) -> None:
        self.prefix_cache.lock_handle(handle, unlock=True)

    @property
    def available_size(self) -> int:
        """Tokens that can still be allocated: free pages plus evictable cached tokens."""
        return len(self.free_slots) * self.page_size + self.prefix_cache.size_info.evictable_size

    # ------------------------------------------------------------ slots
    def allocate_paged(self, reqs: List[Req]) -> None:
        """Give every request pages for its tokens [cached_len, device_len) in its page-table row.

        A partly filled last page is reused; only whole new pages are taken.
        """
        P = self.page_size
        spans: List[Tuple[int, int, int]] = []
        need = 0
        for r in reqs:
            first, last = _ceil_div(r.cached_len, P), _ceil_div(r.device_len, P)
            if last > first:
                spans.append((r.table_idx, first, last))
                need += last - first
        if need == 0:
            return
        pages = self._take(need)
        slots = (pages[:, None] + np.arange(P, dtype=np.int32)[None, :]).reshape(-1) if P > 1 else pages
        off = 0
        for row, first, last in spans:
            n = (last - first) * P
            self.page_table[row, first * P: last * P] = slots[off: off + n]
            off += n

    def _take(self, n: int) -> np.ndarray:
        if n > len(self.free_slots):
            evicted = self.prefix_cache.evict((n - len(self.free_slots)) * self.page_size)
            self.free_slots = np.concatenate([self.free_slots, evicted[:: self.page_size]])
            if n > len(self.free_slots):
                raise RuntimeError("eviction did not free enough KV pages")
        out, self.free_slots = self.free_slots[:n], self.free_slots[n:]
        return out

    def _free(self, slots: np.ndarray) -> None:
        if len(slots) == 0:
            return
        pages = np.asarray(slots[:: self.page_size], dtype=np.int32)
        if self._pending_free is not None:
            self._pending_free.append(pages)
        else:
            self.free_slots = np.concatenate([self.free_slots, pages])

    @contextmanager
    def lazy_free_region(self):
        """Collect frees inside the block and return them to the free list once at the end."""
        self._pending_free = []
        try:
            yield
        finally:
            pending, self._pending_free = self._pending_free, None
            if pending:
                self.free_slots = np.concatenate([self.free_slots] + pending)

    def cache_req(self, req: Req, *, finished: bool) -> None:
        """Hand the request's computed KV [0, cached_len) to the prefix cache.

        Of the request's slots: [0, old) were borrowed from the cache; [old, dup) turned
        out to be in the tree already (another request inserted them) and are freed;
        [dup, new) now belong to the tree; [new, cached_len) is a partial last page,
        freed when the request finishes and kept by it otherwise.
        """
        ids = req.input_ids[: req.cached_len]
        slots = self.page_table[req.table_idx, : req.cached_len]
        old = req.cache_handle
        dup, new = self.prefix_cache.insert_prefix(ids, slots)
        self.unlock(old)
        self._free(slots[old.cached_len: dup])
        if finished:
            self._free(slots[new.cached_len:])
        else:
            req.cache_handle = new
            self.lock(new)

    def check_integrity(self) -> None:
        self.prefix_cache.check_integrity()
        cached_pages = self.prefix_cache.size_info.total_size // self.page_size
        if len(self.free_slots) + cached_pages != self.num_pages:
            raise RuntimeError(f"free pages {len(self.free_slots)} + cached pages {cached_pages} != {self.num_pages}")
        if self.page_size > 1 and np.any(self.free_slots % self.page_size):
            raise RuntimeError("a free slot is not page aligned")


class TableManager:
    """Page-table rows for running requests and the device pool of each row's newest token.

    The decode input of a request is the token sampled in the previous step, which
    may not have reached the host yet (overlap scheduling), so the sampler writes it
    into ``token_pool[row]`` on the device and the next step gathers from there.
    ``token_pool`` has one extra entry, row ``max_running_req``: the pad row that
    padded CUDA-graph batches read and write.
    """

    def __init__(self, max_running_req: int, page_table: np.ndarray, device: torch.device) -> None:
        self._free_rows = list(range(max_running_req))
        self.page_table = page_table
        self.token_pool = torch.zeros(max_running_req + 1, dtype=torch.int32, device=device)

    @property
    def available_size(self) -> int:
        return len(self._free_rows)

    def allocate(self) -> int:
        return self._free_rows.pop()

    def free(self, row: int) -> None:
        self._free_rows.append(row)


class ChunkedReq(Req):
    """A request whose prompt is only partly computed this step: not sampled, not decoded."""

    def append_host(self, next_token: int) -> None:
        raise RuntimeError("a chunked prefill request is not sampled")

    @property
    def can_decode(self) -> bool:
        return False


@dataclass
class PendingReq:
    uid: int
    input_ids: np.ndarray
    sampling_params: object
    chunked_req: ChunkedReq | None = None

    @property
    def input_len(self) -> int:
        return len(self.input_ids)

    @property
    def output_len(self) -> int:
        return int(self.sampling_params.max_tokens)


@dataclass
class DecodeManager:
    page_size: int
    running_reqs: Set[Req] = field(default_factory=set)

    def filter_reqs(self, reqs) -> None:
        """Add the requests of the batch just built; drop the ones that cannot decode further."""
        self.running_reqs = {r for r in self.running_reqs.union(reqs) if r.can_decode}

    def remove_req(self, req: Req) -> None:
        self.running_reqs.discard(req)

    @property
    def inflight_tokens(self) -> int:
        """KV the running requests may still need, plus one spare page per request."""
        return sum(r.remain_len for r in self.running_reqs) + (self.page_size - 1) * len(self.running_reqs)

    def schedule_next_batch(self) -> Batch | None:
        if not self.running_reqs:
            return None
        return Batch(reqs=sorted(self.running_reqs, key=lambda r: r.uid), phase="decode")

    @property
    def runnable(self) -> bool:
        return bool(self.running_reqs)


class PrefillManager:
    def __init__(self, cache: CacheManager, table: TableManager, decode: DecodeManager) -> None:
        self.cache = cache
        self.table = table
        self.decode = decode
        self.pending_list: List[PendingReq] = []

    def add_one_req(self, uid: int, input_ids: np.ndarray, sampling_params) -> None:
        self.pending_list.append(PendingReq(uid, np.asarray(input_ids, dtype=np.int32), sampling_params))

    @property
    def runnable(self) -> bool:
        return bool(self.pending_list)

    def schedule_next_batch(self, token_budget: int) -> Batch | None:
        """FCFS: admit pending requests while the token budget and the KV reservation allow."""
        if not self.pending_list:
            return None
        budget = token_budget
        reserved = self.decode.inflight_tokens
        reqs: List[Req] = []
        chunked: List[PendingReq] = []
        for pr in self.pending_list:
            if budget <= 0:
                break
            if pr.chunked_req is not None:  # continue a prompt admitted earlier
                c = pr.chunked_req
                handle, row, cached = c.cache_handle, c.table_idx, c.cached_len
            else:
                got = self._admit(pr, reserved)
                if got is None:
                    break
                handle, row = got
                cached = handle.cached_len
            remain = pr.input_len - cached
            chunk = min(budget, remain)
            budget -= chunk
            reserved += remain + pr.output_len
            cls = ChunkedReq if chunk < remain else Req
            req = cls(input_ids=pr.input_ids[: cached + chunk], table_idx=row, cached_len=cached,
                      output_len=pr.output_len, uid=pr.uid, sampling_params=pr.sampling_params,
                      cache_handle=handle)
            pr.chunked_req = req if cls is ChunkedReq else None
            if cls is ChunkedReq:
                chunked.append(pr)
            reqs.append(req)
        if not reqs:
            return None
        self.pending_list = chunked + self.pending_list[len(reqs):]
        return Batch(reqs=reqs, phase="prefill")

    def _admit(self, pr: PendingReq, reserved: int):
        if self.table.available_size == 0:
            return None
        handle = self.cache.match_req(pr.input_ids)
        need = (pr.input_len - handle.cached_len) + pr.output_len
        if need + reserved > self.cache.available_size:
            return None
        self.cache.lock(handle)  # the matched prefix stops being evictable: check again
        if need + reserved > self.cache.available_size:
            self.cache.unlock(handle)
            return None
        row = self.table.allocate()
        if handle.cached_len > 0:
            self.table.page_table[row, : handle.cached_len] = handle.get_matched_indices()
        return handle, row
