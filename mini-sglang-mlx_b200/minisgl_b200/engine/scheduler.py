"""Engine, overlap scheduler and offline LLM front end of the engine harness.

* ``Engine``     python/minisgl_mlx/engine/engine.py:43-117: model, KV pool,
  host page table, global Context, attention backend, greedy sampler.
* ``Scheduler``  scheduler/scheduler.py:75-222: prefill first, else one decode
  step of every running request; KV pages are allocated per batch, the
  attention metadata is prepared on the host, results are appended and
  finished requests release their row and pages (their KV goes to the
  prefix cache).
* ``LLM``        llm.py: ``generate(prompts, sampling_params)`` over the same
  loop, fed from a Python list about one prefill budget at a time.

Overlap scheduling (scheduler.py:87-115) with CUDA streams in place of MLX's
lazy graph: kernel launches are asynchronous, so step t+1 is scheduled,
prepared and launched while the GPU still runs step t; only then does the host
wait for step t's sampled tokens (copied to pinned memory behind an event)
and process them. A decode step reads its input tokens from the device token
pool that the previous step's sampler wrote, so no host round trip sits
between two steps.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import numpy as np
import torch

from ..attention import create_attention_backend, page_table_scatter
from ..attention.base import PinnedStager
from ..core import Batch, Context, Req, SamplingParams, batch_positions_out_loc, set_global_ctx
from ..kvcache import MHAKVCache
from .graph import DecodeGraphs
from .managers import CacheManager, ChunkedReq, DecodeManager, PrefillManager, TableManager
from .model import Qwen3Model, Qwen3Spec

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


@dataclass(frozen=True)
class EngineConfig:
    """Defaults follow engine/config.py:6-21 and scheduler/config.py:13-17; page_size 16 is the
    page size the B200 extend kernel's TMA gather takes (page_size 1 runs the fp32-exact path)."""

    spec: Qwen3Spec
    dtype: str = "bfloat16"
    attention_backend: str = "b200"
    max_running_req: int = 128
    page_size: int = 16
    num_tokens: int = 131072  # KV pool tokens per layer (reference max_kv_tokens)
    max_seq_len: int | None = None
    max_extend_tokens: int = 4096  # prefill token budget per batch (chunked prefill)
    cache_type: str = "radix"
    overlap_scheduling: bool = True
    cuda_graph_max_bs: int = 128  # decode batches up to this size replay CUDA graphs (0: eager)
    # keep a device copy of the page table; CUDA-graph decode steps then build their
    # attention metadata on the device, inside the graph (b2a_decode_metadata)
    device_metadata: bool = True
    # bf16 steps of <= 32 tokens run the layers' projections as b2a_proj launches with the
    # norms, residual adds and SwiGLU fused in (False: cuBLAS + separate kernels throughout)
    fused_proj: bool = True
    seed: int = 42


class Engine:
    def __init__(self, cfg: EngineConfig, device: torch.device | None = None) -> None:
        self.cfg = cfg
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.dtype = _DTYPES[cfg.dtype]
        a = cfg.spec.attn
        self.model = Qwen3Model(cfg.spec, self.dtype, self.device, seed=cfg.seed)
        self.model.fused_proj = self.model.fused_proj and cfg.fused_proj
        P = cfg.page_size
        self.num_tokens = cfg.num_tokens // P * P
        self.kv_cache = MHAKVCache(a.num_layers, self.num_tokens, a.num_kv_heads, a.head_dim, self.dtype,
                                   device=self.device)
        self.max_seq_len = cfg.max_seq_len or min(a.rotary_config.max_position, self.num_tokens)
        # the pool's last page and the page table's last row are reserved for padded
        # CUDA-graph batches: a pad request is one token at the pad slot
        self.num_pages = self.num_tokens // P - 1
        self.pad_slot = self.num_pages * P
        self.pad_row = cfg.max_running_req
        self.page_table = np.zeros((cfg.max_running_req + 1, self.max_seq_len), dtype=np.int32)
        self.page_table[self.pad_row, :P] = self.pad_slot + np.arange(P, dtype=np.int32)
        # device copy, kept current by the scheduler with the slots each step allocates
        self.page_table_dev = torch.from_numpy(self.page_table).to(self.device) if cfg.device_metadata else None
        self.ctx = Context(page_size=cfg.page_size)
        self.ctx.page_table = self.page_table
        self.ctx.kv_cache = self.kv_cache
        self.attn_backend = create_attention_backend(cfg.attention_backend, a, self.kv_cache, self.page_table)
        self.ctx.attn_backend = self.attn_backend
        set_global_ctx(self.ctx)

    def forward_batch(self, batch: Batch) -> torch.Tensor:
        """One forward + greedy sampling; returns the next token of every request (device int32 [B])."""
        with self.ctx.forward_batch(batch):
            logits = self.model(batch.input_ids)
        for r in batch.reqs:
            r.complete_one()  # the host advances as if the step were done (overlap scheduling)
        return torch.argmax(logits, dim=-1).to(torch.int32)

    def shutdown(self) -> None:
        set_global_ctx(None)


@dataclass
class _Step:
    batch: Batch
    host_tokens: torch.Tensor  # pinned int32 [B]
    done: torch.cuda.Event
    start: torch.cuda.Event


class HostScheduler:
    """The host half of the scheduler (scheduler/scheduler.py:75-222 without the forward):
    admission and chunked prefill, page allocation, prefix-cache bookkeeping and the
    processing of sampled tokens. It does no device work, so the same code serves the
    engine and a host-only run (e.g. counting prefix-cache hits of a request partition)."""

    def __init__(self, cfg: EngineConfig, page_table: np.ndarray, num_pages: int,
                 device: torch.device | None = None) -> None:
        self.cfg = cfg
        P = cfg.page_size
        self.table = TableManager(cfg.max_running_req, page_table, device or torch.device("cpu"))
        self.cache = CacheManager(num_pages, P, page_table, cfg.cache_type)
        self.decode = DecodeManager(P)
        self.prefill = PrefillManager(self.cache, self.table, self.decode)
        self.finished_reqs: set = set()
        self.eos_token_ids: set = set()
        self.num_output_tokens = 0
        self.num_prefill_tokens = 0
        self.num_prefix_hit_tokens = 0  # prompt tokens served from the prefix cache
        self.num_steps = {"prefill": 0, "decode": 0}

    def next_batch(self) -> Batch | None:
        """Prefill first, else one decode step of every running request; pages allocated."""
        batch = self.prefill.schedule_next_batch(self.cfg.max_extend_tokens) or self.decode.schedule_next_batch()
        if batch is None:
            return None
        self.cache.allocate_paged(batch.reqs)
        self.num_steps[batch.phase] += 1
        if batch.is_prefill:
            self.num_prefill_tokens += sum(r.extend_len for r in batch.reqs)
            # a request's first chunk starts exactly at its prefix-cache hit
            self.num_prefix_hit_tokens += sum(r.cached_len for r in batch.reqs
                                              if r.cached_len == r.cache_handle.cached_len)
        return batch

    def process_tokens(self, batch: Batch, tokens: Sequence[int]) -> None:
        """Append each request's sampled token; finished requests release their row and pages
        (their KV goes to the prefix cache), a prefilled prompt's KV joins the prefix cache."""
        new_finished = set()
        with self.cache.lazy_free_region():
            for req, tok in zip(batch.reqs, tokens):
                if isinstance(req, ChunkedReq) or req in self.finished_reqs:
                    # a chunk has no meaningful token; a request that finished one step earlier
                    # was already placed into this batch, its extra token is dropped
                    continue
                req.append_host(tok)
                finished = len(req.input_ids) >= req.max_device_len
                if not req.sampling_params.ignore_eos:
                    finished |= tok in self.eos_token_ids
                self.on_token(req, tok, finished)
                self.num_output_tokens += 1
                if finished:
                    self.decode.remove_req(req)
                    self.table.free(req.table_idx)
                    self.cache.cache_req(req, finished=True)
                    new_finished.add(req)
                elif batch.is_prefill:
                    self.cache.cache_req(req, finished=False)  # the prompt's KV joins the prefix cache
        self.finished_reqs = new_finished

    def on_token(self, req: Req, token: int, finished: bool) -> None:
        """Called for every sampled token in order (the offline front end collects them)."""

    @property
    def idle(self) -> bool:
        return not (self.prefill.runnable or self.decode.runnable)


class Scheduler(HostScheduler):
    def __init__(self, cfg: EngineConfig, device: torch.device | None = None) -> None:
        self.engine = Engine(cfg, device)
        super().__init__(cfg, self.engine.page_table, self.engine.num_pages, self.engine.device)
        self._stager = PinnedStager(slots=4)
        self._host_ring = [torch.empty(cfg.max_running_req, dtype=torch.int32, pin_memory=True) for _ in range(4)]
        self._ring_next = 0
        # seconds: host scheduling + input/metadata preparation + launches, host result
        # processing, host blocked on the GPU; GPU time of each phase (events around each step)
        self.timing = {"host_launch": 0.0, "host_process": 0.0, "host_wait": 0.0, "gpu_prefill": 0.0,
                       "gpu_decode": 0.0}
        self.graphs = None
        if cfg.cuda_graph_max_bs > 0:
            self.graphs = DecodeGraphs(self.engine, self.table.token_pool, self.engine.pad_row, self.engine.pad_slot,
                                       min(cfg.cuda_graph_max_bs, cfg.max_running_req))
            self.graphs.capture()

    # ------------------------------------------------------------ one step
    def _schedule_next_batch(self) -> Batch | None:
        batch = self.next_batch()
        if batch is not None:
            self._prepare(batch)
        return batch

    def _prepare(self, batch: Batch) -> None:
        reqs = batch.reqs
        positions, out_loc = batch_positions_out_loc(batch, self.engine.page_table)
        rows = np.array([r.table_idx for r in reqs], dtype=np.int32)
        if batch.is_decode and self.graphs is not None and self.graphs.bucket_for(batch.size) is not None:
            # replayed from a CUDA graph: inputs and metadata go into the bucket's buffers in _forward
            batch.graph_inputs = (rows, np.array([r.device_len for r in reqs], dtype=np.int64), positions, out_loc)
            return
        arrays = [positions, out_loc, rows]
        if batch.is_prefill:
            arrays.append(np.concatenate([r.input_ids[r.cached_len: r.device_len] for r in reqs]).astype(np.int32))
        mirror = self.engine.page_table_dev is not None
        if mirror:
            # page-table entries this step makes valid, for the device copy: a decode
            # token's new slot; a prefill request's whole row so far (its prefix-cache
            # hit was written on the host when it was admitted)
            if batch.is_decode:
                arrays += [rows, positions, out_loc]
            else:
                lens = np.array([r.device_len for r in reqs], dtype=np.int64)
                cols = np.concatenate([np.arange(n, dtype=np.int32) for n in lens.tolist()])
                r_tok = np.repeat(rows, lens)
                arrays += [r_tok, cols, self.engine.page_table[r_tok, cols]]
        dev = self._stager.upload(arrays, self.engine.device)
        if mirror:
            page_table_scatter(self.engine.page_table_dev, *dev[-3:])
        batch.positions, batch.out_loc = dev[0], dev[1]
        batch.rows = dev[2]
        batch.input_ids = dev[3] if batch.is_prefill else self.table.token_pool[dev[2].long()]
        self.engine.attn_backend.prepare_metadata(batch)

    def _forward(self, batch: Batch) -> _Step:
        start = torch.cuda.Event(enable_timing=True)
        start.record()
        gi = getattr(batch, "graph_inputs", None)
        if gi is not None:
            tokens = self.graphs.run(*gi)
            for r in batch.reqs:
                r.complete_one()
            rows_dev = self.graphs.rows[: batch.size]
        else:
            tokens = self.engine.forward_batch(batch)
            rows_dev = batch.rows
        self.table.token_pool[rows_dev.long()] = tokens
        host = self._host_ring[self._ring_next][: batch.size]
        self._ring_next = (self._ring_next + 1) % len(self._host_ring)
        host.copy_(tokens, non_blocking=True)
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.decode.filter_reqs(batch.reqs)
        return _Step(batch, host, ev, start)

    def _process(self, step: _Step | None) -> None:
        if step is None:
            return
        t0 = time.perf_counter()
        step.done.synchronize()
        t1 = time.perf_counter()
        self.timing["host_wait"] += t1 - t0
        self.timing["gpu_" + step.batch.phase] += step.start.elapsed_time(step.done) * 1e-3
        self.process_tokens(step.batch, step.host_tokens.tolist())
        self.timing["host_process"] += time.perf_counter() - t1

    # ------------------------------------------------------------ loops
    def overlap_step(self, last: _Step | None) -> _Step | None:
        """Launch step t+1 while step t runs, then process step t."""
        t0 = time.perf_counter()
        batch = self._schedule_next_batch()
        ongoing = self._forward(batch) if batch is not None else None
        self.timing["host_launch"] += time.perf_counter() - t0
        self._process(last)
        return ongoing

    def normal_step(self) -> bool:
        batch = self._schedule_next_batch()
        if batch is not None:
            self._process(self._forward(batch))
        return batch is not None

class LLM(Scheduler):
    """Offline batch generation (reference llm.py): token-id prompts in, token ids out."""

    def __init__(self, cfg: EngineConfig, device: torch.device | None = None) -> None:
        super().__init__(cfg, device)
        self._queue: List[Tuple[int, np.ndarray, SamplingParams]] = []
        self._outputs: Dict[int, List[int]] = {}

    def on_token(self, req: Req, token: int, finished: bool) -> None:
        # a request that stopped at EOS does not output the EOS token itself
        if not (finished and not req.sampling_params.ignore_eos and token in self.eos_token_ids):
            self._outputs[req.uid].append(token)

    def _feed(self) -> None:
        """Deliver about one prefill budget of queued prompts (requests trickle in, as in llm.py)."""
        budget = 0
        while self._queue and budget < self.cfg.max_extend_tokens:
            uid, ids, sp = self._queue.pop(0)
            if len(ids) == 0 or len(ids) >= self.engine.max_seq_len:
                raise ValueError(f"request {uid}: prompt length {len(ids)} outside [1, {self.engine.max_seq_len})")
            if sp.max_tokens > self.engine.max_seq_len - len(ids):
                sp = SamplingParams(sp.temperature, sp.top_k, sp.top_p, sp.ignore_eos,
                                    self.engine.max_seq_len - len(ids))
            budget += len(ids)
            self.prefill.add_one_req(uid, ids, sp)

    def generate(self, prompts: Sequence[Sequence[int]],
                 sampling_params: SamplingParams | Sequence[SamplingParams]) -> List[Dict[str, List[int]]]:
        if isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(prompts)
        if any(not sp.is_greedy for sp in sampling_params):
            raise ValueError("the engine harness samples greedily only")
        self._queue = [(i, np.asarray(p, dtype=np.int32), sp) for i, (p, sp) in
                       enumerate(zip(prompts, sampling_params, strict=True))]
        self._outputs = {i: [] for i in range(len(prompts))}
        last = None
        stalled = 0
        while True:
            self._feed()
            if self.idle and last is None and not self._queue:
                break
            in_flight = last is not None
            if self.cfg.overlap_scheduling:
                last = self.overlap_step(last)
                progressed = last is not None
            else:
                progressed = self.normal_step()
            # nothing launched twice in a row with nothing in flight: a pending request can never fit
            stalled = 0 if (progressed or in_flight or self.decode.runnable) else stalled + 1
            if stalled >= 2:
                raise RuntimeError("no pending request fits the KV pool (prompt + max_tokens > pool)")
        torch.cuda.synchronize(self.engine.device)
        return [{"token_ids": self._outputs[i]} for i in range(len(prompts))]
