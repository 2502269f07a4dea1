"""CUDA graphs of the decode forward, one per batch-size bucket.

A decode step of the harness launches ~16 kernels per layer from Python; at
batch 128 the host needs several milliseconds for that, more than the GPU
needs for the step. The decode forward (token gather from the device token
pool, embeddings, all layers with fused RoPE + KV store and split-KV
attention, final norm, LM head, argmax) is therefore captured once per bucket
of a batch-size ladder and replayed. Per step the host only writes the
bucket's static inputs -- page-table rows, lengths, positions, KV slots.
With the engine's device page table the graph itself applies the new slots
to it and builds the attention metadata from it (b2a_page_table_scatter,
b2a_decode_metadata); without it the host rewrites the metadata in place
(fixed-capacity buffers, see ``B200AttnBackend.alloc_decode_graph_metadata``).
A batch is padded up to its bucket with one-token requests on a reserved pad
row whose page is a reserved pad page of the pool, so padding computes real,
discarded values.
"""

from __future__ import annotations

from typing import Dict, List

import numpy as np
import torch

from ..attention import page_table_scatter
from ..attention.base import PinnedStager
from ..core import Batch

BUCKETS = (1, 2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256)


class DecodeGraphs:
    def __init__(self, engine, token_pool: torch.Tensor, pad_row: int, pad_slot: int, max_batch: int) -> None:
        self.engine = engine
        self.token_pool = token_pool
        self.pad_row = pad_row
        self.pad_slot = pad_slot
        self.buckets: List[int] = [b for b in BUCKETS if b < max_batch] + [max_batch]
        bmax = self.buckets[-1]
        dev = engine.device
        self.rows = torch.full((bmax,), pad_row, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(bmax, dtype=torch.int32, device=dev)
        self.out_loc = torch.full((bmax,), pad_slot, dtype=torch.int32, device=dev)
        self.lens = torch.ones(bmax, dtype=torch.int32, device=dev)
        self.page_table_dev = engine.page_table_dev  # None: metadata built on the host
        self._stager = PinnedStager(slots=4)
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.metas: Dict[int, object] = {}
        self.outs: Dict[int, torch.Tensor] = {}
        self._batches: Dict[int, Batch] = {}

    def bucket_for(self, n: int) -> int | None:
        for b in self.buckets:
            if b >= n:
                return b
        return None

    def capture(self) -> None:
        eng = self.engine
        be = eng.attn_backend
        pages_per_req = -(-eng.max_seq_len // eng.cfg.page_size)
        pool = torch.cuda.graph_pool_handle()
        for b in reversed(self.buckets):  # largest first: smaller graphs reuse its pool blocks
            meta = be.alloc_decode_graph_metadata(b, b * pages_per_req)
            be.fill_decode_graph_metadata(meta, np.full(b, self.pad_row), np.ones(b, dtype=np.int64))
            batch = Batch(reqs=[], phase="decode")
            batch.positions, batch.out_loc, batch.attn_metadata = self.positions[:b], self.out_loc[:b], meta
            rows = self.rows[:b]

            def step():
                if self.page_table_dev is not None:
                    page_table_scatter(self.page_table_dev, rows, batch.positions, batch.out_loc)
                    be.build_decode_metadata_device(meta, self.page_table_dev, rows, self.lens[:b])
                with eng.ctx.forward_batch(batch):
                    logits = eng.model(self.token_pool[rows.long()])
                return torch.argmax(logits, dim=-1).to(torch.int32)

            side = torch.cuda.Stream(eng.device)
            side.wait_stream(torch.cuda.current_stream(eng.device))
            with torch.cuda.stream(side):
                step()  # warm-up outside capture: lazy init, kernel attributes
            torch.cuda.current_stream(eng.device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                out = step()
            self.graphs[b], self.metas[b], self.outs[b], self._batches[b] = g, meta, out, batch
        torch.cuda.synchronize(eng.device)

    def run(self, rows: np.ndarray, lens: np.ndarray, positions: np.ndarray, out_loc: np.ndarray) -> torch.Tensor:
        """Replay the bucket for ``len(rows)`` decode requests; returns their next tokens (device int32)."""
        n = len(rows)
        b = self.bucket_for(n)
        pad = b - n
        rows_p = np.concatenate([rows, np.full(pad, self.pad_row)]).astype(np.int32)
        lens_p = np.concatenate([lens, np.ones(pad, dtype=np.int64)])
        pos_p = np.concatenate([positions, np.zeros(pad, dtype=np.int32)]).astype(np.int32)
        loc_p = np.concatenate([out_loc, np.full(pad, self.pad_slot)]).astype(np.int32)
        if self.page_table_dev is not None:
            self._stager.upload([rows_p, pos_p, loc_p, lens_p.astype(np.int32)], self.engine.device,
                                out=[self.rows[:b], self.positions[:b], self.out_loc[:b], self.lens[:b]])
        else:
            self._stager.upload([rows_p, pos_p, loc_p], self.engine.device,
                                out=[self.rows[:b], self.positions[:b], self.out_loc[:b]])
            self.engine.attn_backend.fill_decode_graph_metadata(self.metas[b], rows_p, lens_p)
        self.graphs[b].replay()
        return self.outs[b][:n]
