"""Prefix caches of the engine harness: radix tree (``radix``) and none (``naive``).

Same contract as python/minisgl_mlx/kvcache/{base,radix_cache,naive_cache}.py:
``match_prefix(ids) -> MatchResult(handle)``, ``lock_handle(handle, unlock)``,
``insert_prefix(ids, slots) -> InsertResult(prefix_len, handle)``,
``evict(n) -> slots`` and ``size_info`` (evictable / protected token counts).

The radix tree stores token runs with their KV slots. With page size P it
matches and inserts whole pages only: a child is found by the first page of
the remaining tokens, and a partial match splits the child at a page boundary
(radix_cache.py:247-268). A node referenced by a running request
(``refs > 0``) is protected; unreferenced leaves are evicted least recently
used first (radix_cache.py:175-199). Recency is a counter bumped on every
walk, so eviction order is deterministic.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Dict, List, NamedTuple, Tuple

import numpy as np

_EMPTY = np.empty(0, dtype=np.int32)


class SizeInfo(NamedTuple):
    evictable_size: int  # tokens no running request references
    protected_size: int  # tokens referenced by at least one request

    @property
    def total_size(self) -> int:
        return self.evictable_size + self.protected_size


@dataclass(frozen=True)
class PrefixHandle:
    """A matched (or inserted) prefix: its length and the tree node that ends it."""

    cached_len: int
    node: "_Node | None" = None

    def get_matched_indices(self) -> np.ndarray:
        """KV slots of the first ``cached_len`` tokens, root to node."""
        parts: List[np.ndarray] = []
        n = self.node
        while n is not None and n.parent is not None:
            parts.append(n.value)
            n = n.parent
        if not parts:
            return _EMPTY
        return np.concatenate(parts[::-1])


class MatchResult(NamedTuple):
    handle: PrefixHandle


class InsertResult(NamedTuple):
    cached_len: int  # tokens already in the tree before the insert (the caller's copies are redundant)
    handle: PrefixHandle


class _Node:
    __slots__ = ("children", "parent", "key", "value", "refs", "last_use")

    def __init__(self, parent: "_Node | None", key: np.ndarray, value: np.ndarray, last_use: int) -> None:
        self.children: Dict[object, _Node] = {}
        self.parent = parent
        self.key = key
        self.value = value
        self.refs = 0
        self.last_use = last_use

    def __lt__(self, other: "_Node") -> bool:
        return self.last_use < other.last_use


class RadixPrefixCache:
    def __init__(self, page_size: int = 1) -> None:
        self.page_size = int(page_size)
        self.root = _Node(None, _EMPTY, _EMPTY, 0)
        self.root.refs = 1  # never evicted
        self.evictable_size = 0
        self.protected_size = 0
        self._clock = 0

    # ------------------------------------------------------------ helpers
    def _child_key(self, ids: np.ndarray) -> object:
        if self.page_size == 1:
            return int(ids[0])
        return ids[: self.page_size].tobytes()

    def _attach(self, parent: _Node, node: _Node) -> None:
        node.parent = parent
        parent.children[self._child_key(node.key)] = node

    def _split(self, node: _Node, pos: int) -> _Node:
        """Cut ``node`` after ``pos`` tokens; return the new upper part (the lower part keeps ``node``)."""
        parent = node.parent
        upper = _Node(None, node.key[:pos], node.value[:pos], node.last_use)
        upper.refs = node.refs
        self._attach(parent, upper)  # replaces node under the same first-page key
        node.key, node.value = node.key[pos:], node.value[pos:]
        self._attach(upper, node)
        return upper

    def _walk(self, ids: np.ndarray) -> Tuple[_Node, int]:
        """Longest page-aligned match of ``ids``; splits a partially matched node."""
        P = self.page_size
        self._clock += 1
        node, done, n = self.root, 0, len(ids)
        while n - done >= P:
            child = node.children.get(self._child_key(ids[done:]))
            if child is None:
                break
            rest = ids[done: done + len(child.key)]
            diff = np.flatnonzero(child.key[: len(rest)] != rest)
            common = int(diff[0]) if diff.size else len(rest)
            common -= common % P
            child.last_use = self._clock
            done += common
            if common < len(child.key):
                node = self._split(child, common) if common > 0 else node
                break
            node = child
        return node, done

    # ------------------------------------------------------------ contract
    def match_prefix(self, input_ids: np.ndarray) -> MatchResult:
        node, n = self._walk(np.asarray(input_ids, dtype=np.int32))
        return MatchResult(PrefixHandle(n, node))

    def lock_handle(self, handle: PrefixHandle, unlock: bool = False) -> None:
        node = handle.node
        while node is not None and node.parent is not None:
            if unlock:
                node.refs -= 1
                assert node.refs >= 0, "unbalanced unlock"
                if node.refs == 0:
                    self.evictable_size += len(node.key)
                    self.protected_size -= len(node.key)
            else:
                if node.refs == 0:
                    self.evictable_size -= len(node.key)
                    self.protected_size += len(node.key)
                node.refs += 1
            node = node.parent

    def insert_prefix(self, input_ids: np.ndarray, indices: np.ndarray) -> InsertResult:
        P = self.page_size
        n = len(input_ids) - len(input_ids) % P
        ids = np.asarray(input_ids[:n], dtype=np.int32)
        slots = np.asarray(indices[:n], dtype=np.int32)
        node, matched = self._walk(ids)
        if matched < n:
            leaf = _Node(None, ids[matched:].copy(), slots[matched:].copy(), self._clock)
            self._attach(node, leaf)
            self.evictable_size += n - matched
            node = leaf
        return InsertResult(matched, PrefixHandle(n, node))

    def evict(self, size: int) -> np.ndarray:
        if size <= 0:
            return _EMPTY
        if size > self.evictable_size:
            raise RuntimeError(f"cannot evict {size} tokens, only {self.evictable_size} evictable")
        heap = [n for n in self._nodes() if not n.children and n.refs == 0]
        heapq.heapify(heap)
        out: List[np.ndarray] = []
        freed = 0
        while freed < size:
            node = heapq.heappop(heap)
            parent = node.parent
            del parent.children[self._child_key(node.key)]
            out.append(node.value)
            freed += len(node.key)
            self.evictable_size -= len(node.key)
            if parent.parent is not None and not parent.children and parent.refs == 0:
                heapq.heappush(heap, parent)
        return np.concatenate(out)

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(self.evictable_size, self.protected_size)

    def _nodes(self) -> List[_Node]:
        out, stack = [], list(self.root.children.values())
        while stack:
            n = stack.pop()
            out.append(n)
            stack.extend(n.children.values())
        return out

    def check_integrity(self) -> None:
        ev = sum(len(n.key) for n in self._nodes() if n.refs == 0)
        pr = sum(len(n.key) for n in self._nodes() if n.refs > 0)
        if (ev, pr) != (self.evictable_size, self.protected_size):
            raise RuntimeError(f"radix sizes ({ev}, {pr}) != recorded ({self.evictable_size}, {self.protected_size})")


class NaivePrefixCache:
    """Caches nothing (reference kvcache/naive_cache.py): every match has length 0."""

    def __init__(self, page_size: int = 1) -> None:
        self.page_size = page_size

    def match_prefix(self, input_ids: np.ndarray) -> MatchResult:
        return MatchResult(PrefixHandle(0))

    def lock_handle(self, handle: PrefixHandle, unlock: bool = False) -> None:
        pass

    def insert_prefix(self, input_ids: np.ndarray, indices: np.ndarray) -> InsertResult:
        return InsertResult(0, PrefixHandle(0))

    def evict(self, size: int) -> np.ndarray:
        if size > 0:
            raise RuntimeError("the naive prefix cache holds nothing to evict")
        return _EMPTY

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(0, 0)

    def check_integrity(self) -> None:
        pass


SUPPORTED_PREFIX_CACHES = {"radix": RadixPrefixCache, "naive": NaivePrefixCache}


def create_prefix_cache(kind: str, page_size: int):
    if kind not in SUPPORTED_PREFIX_CACHES:
        raise ValueError(f"unknown cache type {kind!r}, supported: {list(SUPPORTED_PREFIX_CACHES)}")
    return SUPPORTED_PREFIX_CACHES[kind](page_size)
