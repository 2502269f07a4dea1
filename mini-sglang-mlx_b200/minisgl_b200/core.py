"""Contract types the attention path reads, with the reference's field names.

Mirrors python/minisgl_mlx/core.py:42-158: the three request lengths
(cached_len / device_len / max_device_len), the per-step Batch fields
(positions, out_loc, attn_metadata) and the global Context that AttentionLayer
reads. Tests and the bench fill them directly; for end-to-end runs the engine
harness (``minisgl_b200.engine``) is the scheduler that fills them. Tensors
here are torch tensors on the GPU (positions/out_loc int32 [T]); the page
table stays a host numpy array, as in the reference.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any, List, Literal

import numpy as np


@dataclass(eq=False)
class Req:
    """One running request (reference core.py:42-96).

    input_ids   [ prompt ............ | generated ... ]
                0      cached_len   device_len   max_device_len
    Tokens [cached_len, device_len) are computed by the next forward.
    """

    input_ids: np.ndarray
    table_idx: int
    cached_len: int
    output_len: int
    uid: int = 0
    sampling_params: Any = None  # SamplingParams (engine harness)
    cache_handle: Any = None  # prefix-cache handle of the matched / inserted prefix

    def __post_init__(self) -> None:
        self.device_len = len(self.input_ids)
        self.max_device_len = len(self.input_ids) + self.output_len
        assert 0 <= self.cached_len < self.device_len <= self.max_device_len

    @property
    def extend_len(self) -> int:
        return self.device_len - self.cached_len

    @property
    def remain_len(self) -> int:
        return self.max_device_len - self.device_len

    @property
    def can_decode(self) -> bool:
        return self.remain_len > 0

    def complete_one(self) -> None:
        self.cached_len = self.device_len
        self.device_len += 1

    def append_host(self, next_token: int) -> None:
        self.input_ids = np.append(self.input_ids, np.int32(next_token))


@dataclass
class SamplingParams:
    """reference core.py:25-39. The engine harness samples greedily (argmax)."""

    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    ignore_eos: bool = False
    max_tokens: int = 1024

    @property
    def is_greedy(self) -> bool:
        return (self.temperature <= 0.0 or self.top_k == 1) and self.top_p == 1.0


@dataclass
class Batch:
    """reference core.py:99-120."""

    reqs: List[Req]
    phase: Literal["prefill", "decode"]
    input_ids: Any = field(default=None, init=False)
    positions: Any = field(default=None, init=False)  # torch int32 [T] (device)
    out_loc: Any = field(default=None, init=False)  # torch int32 [T] (device)
    rows: Any = field(default=None, init=False)  # torch int32 [B] page-table rows (engine harness)
    attn_metadata: Any = field(default=None, init=False)

    @property
    def is_prefill(self) -> bool:
        return self.phase == "prefill"

    @property
    def is_decode(self) -> bool:
        return self.phase == "decode"

    @property
    def size(self) -> int:
        return len(self.reqs)


@dataclass
class Context:
    """reference core.py:123-145. page_table is token-granular even for page_size > 1."""

    page_size: int
    page_table: np.ndarray = field(init=False)
    kv_cache: Any = field(init=False)
    attn_backend: Any = field(init=False)
    _batch: Batch | None = field(default=None, init=False)

    @property
    def batch(self) -> Batch:
        assert self._batch is not None, "No active batch in context"
        return self._batch

    @contextmanager
    def forward_batch(self, batch: Batch):
        assert self._batch is None, "Nested forward_batch is not allowed"
        try:
            self._batch = batch
            yield
        finally:
            self._batch = None


_GLOBAL_CTX: Context | None = None


def set_global_ctx(ctx: Context | None) -> None:
    global _GLOBAL_CTX
    _GLOBAL_CTX = ctx


def get_global_ctx() -> Context:
    assert _GLOBAL_CTX is not None, "Global context is not set"
    return _GLOBAL_CTX


def batch_positions_out_loc(batch: Batch, page_table: np.ndarray):
    """Host computation of positions / out_loc (reference scheduler/scheduler.py:155-158).

    positions = concat(arange(cached_len, device_len)); out_loc = page_table[rows, positions].
    Returns int32 numpy arrays.
    """
    reqs = batch.reqs
    positions = np.concatenate(
        [np.arange(r.cached_len, r.device_len, dtype=np.int32) for r in reqs]
    ).astype(np.int32)
    rows = np.repeat(np.array([r.table_idx for r in reqs]), [r.extend_len for r in reqs])
    out_loc = page_table[rows, positions].astype(np.int32)
    return positions, out_loc
