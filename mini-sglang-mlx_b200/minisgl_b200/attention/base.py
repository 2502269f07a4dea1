"""Attention backend interface and host-side metadata builders.

Mirrors python/minisgl_mlx/attention/base.py:49-105: ``prepare_metadata(batch)``
runs on the host before the forward and stores the per-batch indices in
``batch.attn_metadata``; ``forward(q, k, v, layer_id, batch)`` dispatches on
the batch phase. The prefill metadata keeps the reference's ``last_indices``
and ``q_offsets`` fields (models/transformer.py:112 reads ``last_indices``).

Index metadata is built with numpy on the host exactly as the reference does
(it owns a host page table), then shipped to the device in ONE pinned
host-to-device copy per batch (``PinnedStager``). Copies are stream-ordered
and every staging buffer is guarded by a CUDA event, so a batch prepared while
the previous one still runs never overwrites indices in flight.
"""

from __future__ import annotations

import os
from abc import ABC, abstractmethod
from typing import List, Sequence, Tuple

import numpy as np
import torch

CHECK_METADATA = os.environ.get("MINISGL_B200_CHECK", "0") == "1"


def paged_kv_indices(
    page_table: np.ndarray, rows: np.ndarray, lens: np.ndarray, page_size: int, check: bool = False
) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Page CSR of the first ``lens[b]`` tokens of page-table rows ``rows[b]``.

    Returns int32 ``(kv_indptr [B+1], kv_indices [sum pages], last_page_len [B])``.
    With page_size 1 this is the reference's token CSR (attention/metal.py:145-152):
    ``kv_indices`` is the row-major flatten of the valid page-table entries.
    With page_size P a page id is ``page_table[row, p*P] // P``; the reference's
    allocator hands out P-aligned runs of P consecutive slots
    (scheduler/cache.py:30-31,138-143), which ``check`` verifies.
    """
    rows = np.asarray(rows, dtype=np.int64)
    lens = np.asarray(lens, dtype=np.int64)
    B = lens.shape[0]
    P = int(page_size)
    npages = (lens + P - 1) // P
    kv_indptr = np.zeros(B + 1, np.int32)
    np.cumsum(npages, out=kv_indptr[1:])
    last_page_len = np.where(npages > 0, lens - (npages - 1) * P, 0).astype(np.int32)
    if B == 0 or int(npages.max(initial=0)) == 0:
        return kv_indptr, np.zeros(0, np.int32), last_page_len
    max_pages = int(npages.max())
    valid = np.arange(max_pages)[None, :] < npages[:, None]
    if P == 1:
        kv_indices = page_table[rows[:, None], np.arange(max_pages)[None, :]][valid]
    else:
        cols = np.arange(max_pages) * P
        first = page_table[rows[:, None], cols[None, :]]
        kv_indices = first[valid] // P
        if check:
            _check_page_runs(page_table, rows, lens, P)
    return kv_indptr, np.ascontiguousarray(kv_indices, dtype=np.int32), last_page_len


def _check_page_runs(page_table: np.ndarray, rows: np.ndarray, lens: np.ndarray, P: int) -> None:
    for row, n in zip(rows.tolist(), lens.tolist()):
        slots = page_table[row, :n].astype(np.int64)
        pos = np.arange(n)
        base = slots[pos // P * P]
        if np.any(base % P != 0) or np.any(slots != base + pos % P):
            raise ValueError(f"page table row {row} is not made of aligned runs of {P} slots")


class PinnedStager:
    """Ring of pinned int32 host buffers for one-copy metadata uploads."""

    def __init__(self, slots: int = 4) -> None:
        self._bufs: List[torch.Tensor | None] = [None] * slots
        self._events: List[torch.cuda.Event | None] = [None] * slots
        self._next = 0

    ALIGN = 16  # int32 elements: every array starts on a 64-byte boundary (int4 loads on the device)

    def upload(self, arrays: Sequence[np.ndarray], device: torch.device,
               out: Sequence[torch.Tensor] | None = None) -> List[torch.Tensor]:
        """Copy int32 host arrays to the device in one transfer.

        With ``out``, the arrays land in those existing device tensors instead
        (same sizes; a CUDA graph that captured them reads the new values).
        """
        sizes = [int(a.size) for a in arrays]
        if out is not None:
            if [int(t.numel()) for t in out] != sizes:
                raise ValueError("upload(out=...): array sizes differ from the target tensors")
            return self._upload_into(arrays, out)
        padded = [(n + self.ALIGN - 1) // self.ALIGN * self.ALIGN for n in sizes]
        total = max(self.ALIGN, sum(padded))
        slot = self._next
        self._next = (self._next + 1) % len(self._bufs)
        ev = self._events[slot]
        if ev is not None:
            ev.synchronize()  # the copy that last read this buffer has finished
        buf = self._bufs[slot]
        if buf is None or buf.numel() < total:
            buf = torch.empty(max(total, 2 * (0 if buf is None else buf.numel())), dtype=torch.int32,
                              pin_memory=True)
            self._bufs[slot] = buf
        host = buf.numpy()
        off = 0
        for a, n, pn in zip(arrays, sizes, padded):
            host[off:off + n] = np.asarray(a, dtype=np.int32).reshape(-1)
            host[off + n:off + pn] = 0
            off += pn
        dev = torch.empty(total, dtype=torch.int32, device=device)
        dev.copy_(buf[:total], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._events[slot] = ev
        out, off = [], 0
        for n, pn in zip(sizes, padded):
            out.append(dev[off:off + n])
            off += pn
        return out

    def _upload_into(self, arrays: Sequence[np.ndarray], out: Sequence[torch.Tensor]) -> List[torch.Tensor]:
        staged = self.upload(arrays, out[0].device)
        for dst, src in zip(out, staged):
            dst.copy_(src.view(dst.shape), non_blocking=True)
        return list(out)


class BaseAttnBackend(ABC):
    """reference attention/base.py:77-103."""

    def __init__(self, config, kv_cache, page_table: np.ndarray) -> None:
        self.config = config
        self.kv_cache = kv_cache
        self.page_table = page_table
        self.scale = config.head_dim ** -0.5

    def prepare_metadata(self, batch) -> None:
        if batch.is_prefill:
            batch.attn_metadata = self._prepare_prefill(batch)
        else:
            batch.attn_metadata = self.prepare_decode(batch)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_id: int, batch) -> torch.Tensor:
        """q ``[T, Hq, D]``, k/v ``[T, Hkv, D]`` (already stored in the pool) -> o ``[T, Hq, D]``."""
        if batch.is_prefill:
            return self._forward_prefill(q, k, v, layer_id, batch.attn_metadata)
        return self.forward_decode(q, layer_id, batch.attn_metadata)

    @abstractmethod
    def prepare_decode(self, batch): ...

    @abstractmethod
    def forward_decode(self, q: torch.Tensor, layer_id: int, metadata) -> torch.Tensor: ...

    @abstractmethod
    def _prepare_prefill(self, batch): ...

    @abstractmethod
    def _forward_prefill(self, q, k, v, layer_id: int, meta) -> torch.Tensor: ...
