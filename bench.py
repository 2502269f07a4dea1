#!/usr/bin/env python
"""Benchmark of the B200 attention backend (decode hot path).

Headline metric: decode-attention HBM GB/s. One step = one decode
batch of config 2 through all 28 layers of Qwen3-0.6B attention: per layer the
fused RoPE + KV store of the B new tokens and paged split-KV decode attention
over the cached context (AttentionLayer.__call__, reference layers.py:103-111).

  value  = algorithmic bytes of the step / device time, inputs resident in HBM
           (each layer's KV working set, ~560 MB, exceeds the 126 MB L2); the
           28 layers replay as one CUDA graph
  e2e    = the same metric through the public API with HOST buffers: per step
           the decode metadata is rebuilt on the host (numpy + plan) and copied
           into the graph's metadata buffers, then one graph replays the H2D
           of every layer's q/k/v from pinned memory, the 28 AttentionLayer
           calls and a D2H read of every layer's output (copies of other layers
           overlap each layer's attention)
  roofline: one decode call (one decode_kernel launch, split requests merged
           inside it) per launch, CUDA events; traffic from the committed ncu
           summary when it was captured on the same decode sources
  cpu_baseline: the CPU oracle port (torch, naive gather + masked SDPA) on one
           layer of the same batch (rank 0, N = 1 only)
  extend_config3 / decode_config5 / e2e_offline_config4: the other configurations
           (tcgen05 extend TFLOP/s with the fused RoPE + store's GB/s, long-context
           decode GB/s, end-to-end output tok/s of the engine harness)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
N > 1 is launched by torchrun: every rank runs its own config-2 batch on its
own GPU (request-partitioned weak scaling, no data-path collective).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "mini-sglang-mlx_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode-attn HBM GB/s (% of peak) + end-to-end output tok/s at 1/2/4/8 B200"
UNIT = "GB/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="decode layers per step (default 28 = config 2); fewer only for profiling captures")
    ap.add_argument("--no-extend", action="store_true", help="skip the config-3 extend measurement")
    ap.add_argument("--no-config5", action="store_true", help="skip the config-5 long-context decode measurement")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 end-to-end offline measurement")
    ap.add_argument("--no-page1", action="store_true", help="skip the page-size-1 decode measurement")
    ap.add_argument("--c4-requests", type=int, default=None,
                    help="config 4 with only its first N requests (one rank's share at N = 256/world)")
    ap.add_argument("--no-config4-shared", action="store_true", help="skip the shared-prefix config-4 line")
    ap.add_argument("--proj-sweep", type=str, default=None, metavar="ROWS",
                    help="only time the 28 layers' projections of Qwen3-0.6B at these token counts "
                         "(comma list), fused b2a_proj against cuBLAS + b2a_rmsnorm + b2a_swiglu")
    ap.add_argument("--decode-sweep", type=str, default=None, metavar="BATCHES",
                    help="only time one decode call of config-2 shapes at these batch sizes (comma list)")
    ap.add_argument("--no-fused-proj", action="store_true",
                    help="config 4 with the unfused projections (cuBLAS GEMMs + separate norm / SwiGLU kernels)")
    ap.add_argument("--c5-requests", type=int, default=None,
                    help="config 5 with only its first N requests (profiling captures; default all 1024)")
    return ap.parse_args()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 10 ms while running.

    Read-only: no clock, power or mode setting of the GPU is touched.
    """

    REASONS = {  # NVML clocks-event-reason bits
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        self.gpu = gpu_index
        self.period = period_s
        self.samples = []
        self._stop = None
        self._thread = None
        self._err = None

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self._max = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - report, never fail the bench on telemetry
            self._err = f"nvml unavailable: {e}"
            return
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, rs))
                except Exception:  # noqa: BLE001
                    pass
                time.sleep(self.period)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def stop(self):
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self._err or "no samples"]}
        self._stop.set()
        self._thread.join()
        sms = [s for s, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": self._max,
                "reasons": reasons, "samples": len(sms), "source": "nvml 10 ms"}


# ------------------------------------------------------------------ workload
def decode_bytes(lens: np.ndarray, P: int, Hq: int, Hkv: int, D: int, es: int) -> int:
    """Algorithmic bytes of one decode call: K and V rows of every cached token, q, o, page ids."""
    L = int(lens.sum())
    pages = int(((lens + P - 1) // P).sum())
    B = len(lens)
    return L * Hkv * D * es * 2 + 2 * B * Hq * D * es + 4 * pages + 4 * (B + 1)


def rope_store_bytes(T: int, Hq: int, Hkv: int, D: int, es: int) -> int:
    """q,k read+write, v read, k,v pool write, positions + out_loc."""
    return T * (Hq + Hkv) * D * es * 2 + T * Hkv * D * es * 3 + 8 * T


def cpu_sample(lens, page_table, P, Hq, Hkv, D, num_slots, steps, warmup, seed):
    """Time the oracle port (naive gather + masked SDPA, torch CPU fp32 math on bf16 pools)."""
    import torch

    from oracle.cpu_naive import naive_decode_torch

    torch.set_num_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1))
    g = torch.Generator().manual_seed(seed)
    k_pool = torch.randn((num_slots, Hkv, D), generator=g).to(torch.bfloat16)
    v_pool = torch.randn((num_slots, Hkv, D), generator=g).to(torch.bfloat16)
    q = torch.randn((len(lens), Hq, D), generator=g).to(torch.bfloat16)
    rows = np.arange(len(lens))
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        naive_decode_torch(q, k_pool, v_pool, page_table, rows, lens, D ** -0.5)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    per_call = float(np.mean(times))
    gbs = decode_bytes(lens, P, Hq, Hkv, D, 2) / per_call / 1e9
    return gbs, per_call, torch.get_num_threads()


def measure_config5(dev, rank: int, world: int, seed: int, steps: int, n_requests: int | None = None):
    """Config 5: request-partitioned long-context decode at Qwen3-8B attention shape.

    1024 sequences, context log-uniform in [1024, 131072] (sum ~27.4 M tokens),
    32q/8kv/128, bf16, page 16, split-KV. Requests are sharded longest-first
    across the ranks (no collective); each rank holds ONE layer's pool for its
    shard (~112 GB at 1 GPU) and times repeated decode calls over it. Every
    call streams far more than the 126 MB L2, so HBM GB/s is honest. Reported
    per rank-0 plus the job total (sum of bytes / slowest rank).
    """
    import torch
    import torch.distributed as dist

    from minisgl_b200 import MHAKVCache
    from minisgl_b200 import workloads as W
    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.config import qwen3_8b

    c = W.CONFIG5
    cfg = qwen3_8b()
    Hq, Hkv, D, P = cfg.num_qo_heads, cfg.num_kv_heads, cfg.head_dim, c["page_size"]
    lens_all = W.config5_lens(seed=seed)
    if n_requests:
        lens_all = lens_all[:n_requests]
    mine = W.shard_requests(lens_all, world)[rank]
    lens = lens_all[mine]
    rng = np.random.default_rng(seed + 7 * rank)
    pages = int(((lens + P - 1) // P).sum())
    num_slots = (pages + 64) * P
    free_bytes, _ = torch.cuda.mem_get_info(dev)
    need = num_slots * Hkv * D * 2 * 2
    if need > free_bytes - (8 << 30):
        return {"skipped": f"pool of {need / 1e9:.1f} GB does not fit next to the bench's buffers"}
    pb = W.allocate_pages(lens, num_slots, P, rng)
    kv = MHAKVCache(1, num_slots, Hkv, D, torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(seed + 99 * rank)
    kv.k[0].normal_(generator=gen)
    kv.v[0].normal_(generator=gen)
    be = B200AttnBackend(cfg, kv, pb.page_table, page_size=P)
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens)
    q = torch.randn((len(lens), Hq, D), device=dev, generator=gen).to(torch.bfloat16)
    for _ in range(3):
        be.forward_decode(q, 0, meta)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = []
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    clocks.start()
    for _ in range(max(5, min(steps, 20))):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        be.forward_decode(q, 0, meta)
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    nbytes = decode_bytes(pb.lens, P, Hq, Hkv, D, 2)
    stats = torch.tensor([ms], dtype=torch.float64, device=dev)
    work = torch.tensor([float(nbytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(work, op=dist.ReduceOp.SUM)
    peak, kind = measured_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    out = {"metric": "decode-attn HBM GB/s, one layer call per rank", "value": round(float(work.item()) / (stats.item() * 1e-3) / 1e9, 1),
           "unit": "GB/s", "scaling": "strong (1024 requests split across ranks)", "ms_per_call_max_rank": round(stats.item(), 4),
           "rank0": {"requests": int(len(lens)), "sum_ctx_tokens": int(lens.sum()), "bytes_per_call": nbytes,
                     "ms_per_call": round(ms, 4), "achieved": round(gbs, 1), "frac": round(gbs / peak, 4),
                     "n_partials": meta.n_partials, "pool_gb": round(need / 1e9, 1)},
           "roofline": {"bound": "hbm", "kernel": "decode_mma_kernel<4> (mma.sync tensor cores, TMA boxes)",
                        "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 4), "peak_kind": kind},
           "clocks_rank0": clk,
           "config": {"workload": "config5: Qwen3-8B attention (32q/8kv/128), bf16, page 16, 1024 seqs, "
                                  "L log-uniform [1024, 131072], split-KV, request-partitioned",
                      "sum_ctx_tokens_all": int(lens_all.sum())}}
    del kv, be, meta, q
    torch.cuda.empty_cache()
    return out


def measure_decode_page1(dev, seed: int, steps: int, warmup: int):
    """Config-2 decode shapes at the reference's default page size 1 (engine/config.py:12).

    One layer's pool (262144 slots, 16q/8kv/128, bf16), B = 128 requests with L ~ U[100, 2048]
    from the config-2 generator. Two slot layouts: a seeded random permutation of the pool
    (every token on its own slot, the worst case), and allocator order (a fresh
    page-size-1 free list hands each prompt one run of consecutive slots,
    scheduler/cache.py:28-72). Each call streams ~560 MB > L2.
    """
    import torch

    from minisgl_b200 import MHAKVCache
    from minisgl_b200 import workloads as W
    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.config import qwen3_0_6b

    cfg = qwen3_0_6b()
    Hq, Hkv, D = cfg.num_qo_heads, cfg.num_kv_heads, cfg.head_dim
    c = W.CONFIG2
    N = c["num_slots"]
    lens = W.config2_batch(seed=seed).lens
    kv = MHAKVCache(1, N, Hkv, D, torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(seed)
    kv.k[0].normal_(generator=gen)
    kv.v[0].normal_(generator=gen)
    q = torch.randn((len(lens), Hq, D), device=dev, generator=gen).to(torch.bfloat16)
    peak, kind = measured_peaks()
    nbytes = decode_bytes(lens, 1, Hq, Hkv, D, 2)
    out = {"metric": "decode-attn HBM GB/s at page size 1 (one layer call)", "unit": "GB/s",
           "bytes_per_call": nbytes, "config": {"workload": "config2 shapes at page size 1: B=128, L~U[100,2048], "
                                                             "16q/8kv/128, bf16, 262144-slot pool", "sum_ctx_tokens": int(lens.sum())}}
    rng = np.random.default_rng(seed + 5)
    layouts = {"random_slots": W.permutation_slots(lens, N, rng),
               "allocator_order": W.allocate_pages(lens, N, 1, rng)}
    # allocator order: consecutive runs in request order (a fresh free list), not shuffled
    alloc = layouts["allocator_order"]
    off = 0
    for b, L in enumerate(lens.tolist()):
        alloc.page_table[b, :L] = np.arange(off, off + L, dtype=np.int32)
        off += L
    for name, pb in layouts.items():
        be = B200AttnBackend(cfg, kv, pb.page_table, page_size=1)
        meta = be.decode_metadata_from_lens(pb.rows, pb.lens)
        for _ in range(max(warmup, 3)):
            be.forward_decode(q, 0, meta)
        torch.cuda.synchronize()
        evs = []
        for _ in range(max(steps, 20)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            be.forward_decode(q, 0, meta)
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"value": round(gbs, 1), "ms_per_call": round(ms, 4),
                     "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(gbs / peak, 4), "peak_kind": kind},
                     "kernel": "decode_kernel (1-D bulk copies of slot runs)"}
        del be, meta
    out["value"] = out["random_slots"]["value"]
    del kv, q
    torch.cuda.empty_cache()
    return out


def measure_e2e_offline(dev, rank: int, world: int, seed: int, shared: bool = False, n_requests: int | None = None,
                        fused_proj: bool = True):
    """Config 4: end-to-end offline generation through the engine harness (output tok/s).

    Random-init Qwen3-0.6B (bf16), 256 prompts of U[100,1024] random token ids,
    output U[100,1024] tokens each (ignore_eos, greedy), at most 128 running
    requests, chunked prefill of 4096 tokens, radix prefix cache, overlap
    scheduling, page 16, 131072 KV tokens per layer. Wall time around
    ``LLM.generate`` as benchmark/offline.py:45-48 measures it, after a short
    warm-up generation. Under torchrun the requests are partitioned by the
    prefix-affinity router (engine/router.py: first-page groups, placed
    longest-first) and the job throughput is all outputs / slowest rank.
    Decode steps of <= 32 requests run the layers' projections as b2a_proj
    launches (norm, residual adds and SwiGLU fused) unless ``fused_proj`` is off.
    """
    import time

    import torch
    import torch.distributed as dist

    from minisgl_b200 import workloads as W
    from minisgl_b200.core import SamplingParams
    from minisgl_b200.engine import LLM, EngineConfig, qwen3_0_6b_spec

    from minisgl_b200.engine.router import route_requests

    if shared:
        # 16 system prompts of U[512, 2048] tokens, each starting 16 requests
        c = W.CONFIG4_SHARED
        prompts_all, outs_all, _ = W.config4_shared_workload(seed=seed)
    else:
        c = W.CONFIG4
        prompts_all, outs_all = W.config4_workload(seed=seed)
    if n_requests:
        prompts_all, outs_all = prompts_all[:n_requests], outs_all[:n_requests]
    cost = np.array([len(p) for p in prompts_all]) + outs_all
    mine = route_requests(prompts_all, cost, world, page_size=c["page_size"])[rank]
    prompts = [prompts_all[i] for i in mine]
    outs = [int(outs_all[i]) for i in mine]
    cfg = EngineConfig(spec=qwen3_0_6b_spec(), dtype="bfloat16", max_running_req=c["max_running_req"],
                       page_size=c["page_size"], num_tokens=c["num_tokens"], max_extend_tokens=c["max_extend_tokens"],
                       fused_proj=fused_proj)
    with torch.cuda.device(dev):
        llm = LLM(cfg, device=dev)
        rng = np.random.default_rng(seed + 1)
        llm.generate([rng.integers(0, 10000, 16).astype(np.int32) for _ in range(4)],
                     SamplingParams(max_tokens=16, ignore_eos=True))
        llm.num_output_tokens = llm.num_prefill_tokens = llm.num_prefix_hit_tokens = 0
        llm.num_steps = {"prefill": 0, "decode": 0}
        llm.timing = {k: 0.0 for k in llm.timing}
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        res = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in outs])
        elapsed = time.perf_counter() - t0
        assert [len(r["token_ids"]) for r in res] == outs
        llm.cache.check_integrity()
        stats = torch.tensor([elapsed], dtype=torch.float64, device=dev)
        tot = torch.tensor([float(sum(outs)), float(llm.num_prefix_hit_tokens), float(llm.num_prefill_tokens)],
                           dtype=torch.float64, device=dev)
        hits_per_rank = torch.zeros(world, dtype=torch.float64, device=dev)
        hits_per_rank[rank] = float(llm.num_prefix_hit_tokens)
        if world > 1:
            dist.all_reduce(stats, op=dist.ReduceOp.MAX)
            dist.all_reduce(tot, op=dist.ReduceOp.SUM)
            dist.all_reduce(hits_per_rank, op=dist.ReduceOp.SUM)
        tps = tot[0].item() / stats.item()
        name = "config 4, shared prefixes" if shared else "config 4"
        out = {"metric": f"end-to-end output tok/s (offline, {name})", "value": round(tps, 1),
               "unit": "tok/s", "higher_is_better": True, "scaling": "strong (256 requests split across ranks)",
               # the reference's published figure for this workload shape (README.md:84, Apple M5 Ultra,
               # Metal attention + overlap, real weights, temperature 0.6)
               "vs_published": {"value": 4427.0, "hardware": "Apple M5 Ultra (Metal)", "ratio": round(tps / 4427.0, 2)},
               "wall_s_max_rank": round(stats.item(), 3),
               "prefix_hit_tokens_all": int(tot[1].item()), "prefill_tokens_all": int(tot[2].item()),
               "prefix_hit_tokens_per_rank": [int(x) for x in hits_per_rank.tolist()],
               "rank0": {"requests": len(outs), "output_tokens": int(sum(outs)), "wall_s": round(elapsed, 3),
                         "prefill_tokens": llm.num_prefill_tokens, "prefix_hit_tokens": llm.num_prefix_hit_tokens,
                         "prefill_steps": llm.num_steps["prefill"], "decode_steps": llm.num_steps["decode"],
                         "gpu_ms_per_decode_step": round(1e3 * llm.timing["gpu_decode"] / max(1, llm.num_steps["decode"]), 4),
                         "time_s": {k: round(v, 3) for k, v in llm.timing.items()},
                         "fused_proj_steps_le_32": llm.engine.model.fused_proj,
                         "kv_pool_gb": round(llm.engine.kv_cache.nbytes / 1e9, 2),
                         "model_gb": round(llm.engine.model.nbytes / 1e9, 2)},
               "config": {"workload": ("config4 with shared prefixes: 16 system prompts U[512,2048] x 16 requests, "
                                       "user part U[100,1024], outputs U[100,1024]; random-init Qwen3-0.6B bf16, "
                                       "concurrency 128, greedy, ignore_eos, radix on, overlap on, chunked prefill 4096, "
                                       "page 16, 262144 KV tokens; routed by first-page prefix affinity")
                           if shared else
                           "config4: random-init Qwen3-0.6B bf16, 256 reqs, input/output U[100,1024], "
                           "random ids, concurrency 128, greedy, ignore_eos, radix on, overlap on, "
                           "chunked prefill 4096, page 16, 131072 KV tokens",
                          "input_tokens_all": int(sum(len(p) for p in prompts_all)),
                          "output_tokens_all": int(outs_all.sum())},
               "data": "synthetic (random token ids, random weights)"}
        llm.engine.shutdown()
        del llm
    torch.cuda.empty_cache()
    return out


def extend_flops(prefix: np.ndarray, extend: np.ndarray, Hq: int, D: int) -> float:
    """Causal extend FLOPs: 2 GEMMs x 2 flops x Hq x D x visible keys of every query row."""
    vis = sum(int(e) * int(p) + int(e) * (int(e) + 1) // 2 for p, e in zip(prefix, extend))
    return 4.0 * Hq * D * vis


def extend_executed_flops(prefix: np.ndarray, extend: np.ndarray, Hq: int, Hkv: int, D: int) -> float:
    """FLOPs the tcgen05 extend kernel executes: whole 128-row tiles x whole 128-key blocks.

    A work item is two tiles of 128/G query tokens (G query heads each) of one request;
    tile t runs over every 128-key block up to the last key visible to its last row.
    """
    G = Hq // Hkv
    TT, KB = 128 // G, 128
    blocks = 0
    for p, e in zip(prefix, extend):
        p, e = int(p), int(e)
        for tb in range(0, e, 2 * TT):
            nq = min(e - tb, 2 * TT)
            for t, nqt in enumerate((min(nq, TT), max(0, nq - TT))):
                if nqt:
                    blocks += (min(p + e, p + tb + t * TT + nqt) + KB - 1) // KB
    # per block: S = Q K^T and O += P V, each 2 x 128 x 128 x D flops, for every kv head
    return float(blocks) * Hkv * 2 * (2 * 128 * KB * D)


def measure_extend(dev, seed: int, steps: int, warmup: int, page_size: int | None = None,
                   allocator_order: bool = False):
    """Config 3: 32 ragged requests with a cached radix prefix, fused RoPE+store then extend attention.

    page_size None is config 3's page size 16 (the tcgen05 kernel reads the pool directly);
    page_size 1 is the reference's default: the tcgen05 kernel reads the keys in groups of
    16 (b2a_extend_groups), each group in place when its slots are one run of consecutive
    slots, else from a staging pool the backend packs it into (b2a_pack_kv), both inside
    the timed call. The page-size-1 slots are a seeded random permutation (every group
    packed, the worst case) or, with ``allocator_order``, what a fresh free list hands out
    (scheduler/cache.py:28-72): every prefix one run, then every request's new tokens one run.
    """
    import torch

    from minisgl_b200 import MHAKVCache
    from minisgl_b200 import workloads as W
    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.config import qwen3_0_6b
    from minisgl_b200.layers import RotaryEmbedding

    cfg = qwen3_0_6b()
    Hq, Hkv, D = cfg.num_qo_heads, cfg.num_kv_heads, cfg.head_dim
    eb = W.config3_batch(seed=seed, page_size=page_size)
    pb = eb.paged
    if allocator_order:
        assert pb.page_size == 1
        off = 0
        for b, L in enumerate(eb.prefix.tolist()):
            pb.page_table[b, :L] = np.arange(off, off + L, dtype=np.int32)
            off += L
        for b, (Lp, Le) in enumerate(zip(eb.prefix.tolist(), eb.extend.tolist())):
            pb.page_table[b, Lp:Lp + Le] = np.arange(off, off + Le, dtype=np.int32)
            off += Le
    kv = MHAKVCache(1, pb.num_slots, Hkv, D, torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(seed)
    kv.k[0].normal_(generator=gen)
    kv.v[0].normal_(generator=gen)
    be = B200AttnBackend(cfg, kv, pb.page_table, page_size=pb.page_size)
    meta = be.extend_metadata_from_lens(pb.rows, pb.lens, eb.extend)
    T = int(eb.extend.sum())
    q = torch.randn((T, Hq, D), device=dev, generator=gen).to(torch.bfloat16)
    knew = torch.randn((T, Hkv, D), device=dev, generator=gen).to(torch.bfloat16)
    vnew = torch.randn((T, Hkv, D), device=dev, generator=gen).to(torch.bfloat16)
    pos = np.concatenate([np.arange(p, p + e, dtype=np.int32) for p, e in zip(eb.prefix, eb.extend)])
    rows = np.repeat(pb.rows, eb.extend)
    loc = pb.page_table[rows, pos].astype(np.int32)
    pos_t, loc_t = torch.from_numpy(pos).to(dev), torch.from_numpy(loc).to(dev)
    rope = RotaryEmbedding(cfg.rotary_config, device=dev)
    for _ in range(max(warmup, 3)):
        rope.rope_store_(q, knew, vnew, pos_t, loc_t, kv, 0)
        be._forward_prefill(q, None, None, 0, meta)
    torch.cuda.synchronize()
    evs, revs = [], []
    # at least 50 calls (~13 ms) so that the clock sampler sees the timed region
    n_iter = max(steps, 50)
    clocks = ClockSampler(dev.index if dev.index is not None else 0)
    clocks.start()
    for _ in range(n_iter):
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        rope.rope_store_(q, knew, vnew, pos_t, loc_t, kv, 0)
        r1.record()
        revs.append((r0, r1))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        be._forward_prefill(q, None, None, 0, meta)
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    rope_ms = float(np.mean([a.elapsed_time(b) for a, b in revs]))
    rope_bytes = rope_store_bytes(T, Hq, Hkv, D, 2)
    hbm_peak, hbm_kind = measured_peaks()
    flops = extend_flops(eb.prefix, eb.extend, Hq, D)
    peak = 1636.1
    pk = ROOT / "MEASURED_PEAKS.json"
    kind = "fallback"
    if pk.exists():
        peak, kind = float(json.loads(pk.read_text())["bf16_tflops"]), "measured"
    tf = flops / (ms * 1e-3) / 1e12
    from minisgl_b200 import _native as nat

    tile = nat.extend_tile_q(Hq, Hkv, D, nat.B2A_DTYPE_BF16, max(pb.page_size, 16))
    tc = tile == 2 * (128 // (Hq // Hkv))
    packed_share = None
    if meta.group_starts:  # share of the 16-key groups copied to the staging pool
        packed_share = round((meta.pack.n_groups if meta.pack is not None else 0) / max(1, int(meta.kv_indices.numel())), 4)
    # tile-padded work the tensor cores run (partial query tiles, masked key blocks)
    exe = extend_executed_flops(eb.prefix, eb.extend, Hq, Hkv, D) if tc else None
    return {"metric": "extend attention TFLOP/s (causal, visible keys only)", "value": round(tf, 2),
            "unit": "TFLOP/s", "ms_per_call": round(ms, 4), "flops_per_call": flops, "calls_timed": n_iter,
            "executed": None if exe is None else {
                "flops_per_call": exe, "tflops": round(exe / (ms * 1e-3) / 1e12, 2),
                "frac_of_peak": round(exe / (ms * 1e-3) / 1e12 / peak, 4), "useful_share": round(flops / exe, 4)},
            "clocks": clk,
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / peak, 4), "peak_kind": kind + " (bf16 dense, burst)"},
            "config": {"workload": "config3: 32 ragged requests, prefix U[0,4096] page-aligned (+1 unaligned), "
                                   f"extend U[64,512], 16q/8kv/128, bf16, page {pb.page_size}, RoPE theta 1e6 fused store"
                                   + ((" (16-key groups: runs read in place, the rest packed to a staging pool inside "
                                       "the timed call; slots " + ("in allocator order)" if allocator_order
                                                                    else "a random permutation)")) if pb.page_size < 16 else ""),
                       "tokens": T, "sum_prefix": int(eb.prefix.sum()), "tile_q_tokens": tile,
                       "packed_group_share": packed_share,
                       "kernel": "extend_tc2_kernel (tcgen05, 2 x 128-row tiles)" if tile == 2 * (128 // (Hq // Hkv)) else "extend_simt_kernel"},
            # config 3': the fused RoPE + KV store of the same T tokens (HBM-bound)
            "rope_store_config3p": {"metric": "fused RoPE + KV store HBM GB/s", "value": round(rope_bytes / (rope_ms * 1e-3) / 1e9, 1),
                                    "unit": "GB/s", "ms_per_call": round(rope_ms, 4), "bytes_per_call": rope_bytes,
                                    "roofline": {"bound": "hbm", "peak": hbm_peak, "peak_kind": hbm_kind,
                                                 "frac": round(rope_bytes / (rope_ms * 1e-3) / 1e9 / hbm_peak, 4)},
                                    "config": {"tokens": T, "heads": f"{Hq}q/{Hkv}kv x {D}", "dtype": "bf16"}}}


# ------------------------------------------------------------------ shared line pieces
def load_workloads():
    """The seeded workload generators (mini-sglang-mlx_b200/minisgl_b200/workloads.py, numpy only).

    Loaded by file path, so the reference arm gets its batches without importing the
    minisgl_b200 package (whose import loads the CUDA library).
    """
    import importlib.util

    name = "_bench_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "mini-sglang-mlx_b200" / "minisgl_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def warmup_steps(args) -> int:
    """Untimed warm-up steps, the same in both arms (at least 3)."""
    return max(args.warmup, 3)


def config2_config(W, world: int, B: int, sum_ctx: int, layers: int) -> dict:
    """The `config` of the headline line (config 2), identical in both arms."""
    c = W.CONFIG2
    return {
        "workload": "config2: batched paged decode step, Qwen3-0.6B attention x28 layers "
                    "(16q/8kv/128, bf16, page 16, pool 262144 slots/layer, B=128/GPU, L~U[100,2048], "
                    "fragmented pages); per layer fused RoPE+KV store + split-KV decode",
        "global_batch": B * world, "seq_len": f"U[{c['lo']},{c['hi']}]", "parallelism": f"request-partitioned x{world}",
        "l2": "inputs larger than L2 (each layer's ~560 MB KV working set > 126 MB L2)",
        "sum_ctx_tokens_per_gpu": sum_ctx, "layers": layers,
    }


DECODE_PROFILE = ROOT / "profiles" / "decode_kernel_config2.md"
# the sources of the config-2 decode launch (decode_kernel); the tensor-core decode
# (decode_mma.cuh) serves G >= 4 only and is not in the headline roofline
DECODE_SOURCES = ("mini-sglang-mlx_b200/csrc/decode.cuh", "mini-sglang-mlx_b200/csrc/common.cuh")


def decode_sources_digest() -> str:
    """SHA-256 (first 16 hex digits) of the decode kernel's sources, in DECODE_SOURCES order."""
    import hashlib

    h = hashlib.sha256()
    for f in DECODE_SOURCES:
        h.update((ROOT / f).read_bytes())
    return h.hexdigest()[:16]


def decode_traffic():
    """DRAM bytes (read + write) per decode launch from the committed ncu summary.

    profiles/decode_kernel_config2.md carries a line
    ``traffic: <bytes> bytes per launch, decode sources <digest>``; the figure is
    used only when <digest> is the digest of the sources being timed, so a kernel
    change makes it null ("stale") instead of silently wrong.
    """
    import re

    if not DECODE_PROFILE.exists():
        return None, "no ncu summary committed"
    m = re.search(r"traffic: (\d+) bytes per launch, decode sources ([0-9a-f]{16})", DECODE_PROFILE.read_text())
    if not m:
        return None, "ncu summary has no traffic line"
    if m.group(2) != decode_sources_digest():
        return None, f"stale: captured on decode sources {m.group(2)}, timed on {decode_sources_digest()}"
    return int(m.group(1)), f"ncu capture of the decode launch on config-2 layer 0, seed 0, decode sources {m.group(2)}"


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    """The reference arm: the CPU oracle port of the naive decode (the MLX CPU path cannot
    run on this box). Rank 0 alone runs it; the minisgl_b200 package is never imported."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    W = load_workloads()
    c = W.CONFIG2
    pb = W.config2_batch(seed=args.seed)
    steps = args.steps
    warm = warmup_steps(args)
    gbs, per_call, cores = cpu_sample(pb.lens, pb.page_table, pb.page_size, c["Hq"], c["Hkv"], c["D"],
                                      c["num_slots"], steps, warm, args.seed)
    sample = (f"each step is one of the 28 layers of a config-2 step (B={pb.batch_size}, "
              f"sum L={int(pb.lens.sum())}, bf16 pools, naive gather+mask+SDPA in fp32 on {cores} threads); "
              f"GB/s is the same rate for 1 or 28 layers; {steps} timed steps after {warm} warm-up")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(per_call * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config2_config(W, world, pb.batch_size, int(pb.lens.sum()), c["layers"]),
        "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                         "note": "torch CPU restatement of attention/naive.py:36-60; MLX CPU unavailable on this box"},
        "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from minisgl_b200 import (AttentionLayer, Batch, Context, MHAKVCache, Req, set_global_ctx)
    from minisgl_b200 import workloads as W
    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.config import qwen3_0_6b
    from minisgl_b200.core import batch_positions_out_loc

    c = W.CONFIG2
    cfg = qwen3_0_6b()
    Lyr = args.layers or c["layers"]
    Hq, Hkv, D, P, N = cfg.num_qo_heads, cfg.num_kv_heads, cfg.head_dim, c["page_size"], c["num_slots"]
    pb = W.config2_batch(seed=args.seed + 1000 * rank)
    B = pb.batch_size

    kv = MHAKVCache(Lyr, N, Hkv, D, torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(args.seed + 17 * rank)
    for l in range(Lyr):
        kv.k[l].normal_(generator=gen)
        kv.v[l].normal_(generator=gen)
    ctx = Context(page_size=P)
    ctx.page_table = pb.page_table
    ctx.kv_cache = kv
    be = B200AttnBackend(cfg, kv, pb.page_table, page_size=P)
    ctx.attn_backend = be
    set_global_ctx(ctx)
    layers = [AttentionLayer(l, Hq, Hkv, D, cfg.rotary_config) for l in range(Lyr)]

    # decode batch: the new token of request b sits at position lens[b]-1 (its slot is allocated)
    reqs = []
    for b in range(B):
        L = int(pb.lens[b])
        r = Req(np.zeros(L - 1, np.int32), table_idx=int(pb.rows[b]), cached_len=0, output_len=2)
        r.complete_one()  # cached_len = L-1, device_len = L
        reqs.append(r)
    batch = Batch(reqs, "decode")
    pos, loc = batch_positions_out_loc(batch, pb.page_table)
    batch.positions = torch.from_numpy(pos).to(dev)
    batch.out_loc = torch.from_numpy(loc).to(dev)
    be.prepare_metadata(batch)
    meta = batch.attn_metadata

    # per-layer inputs: q [B, Hq, D] contiguous, new k/v rows interleaved [B, 2, Hkv, D]
    q_all = torch.randn((Lyr, B, Hq, D), device=dev, generator=gen).to(torch.bfloat16)
    kv_all = torch.randn((Lyr, B, 2, Hkv, D), device=dev, generator=gen).to(torch.bfloat16)
    views = [(q_all[l], kv_all[l, :, 0], kv_all[l, :, 1]) for l in range(Lyr)]

    dec_events = []

    def step(record=False):
        with ctx.forward_batch(batch):
            for l in range(Lyr):
                q, k, v = views[l]
                layers[l].rotary.rope_store_(q, k, v, batch.positions, batch.out_loc, kv, l)
                if record:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    be.forward(q, k, v, l, batch)
                    e1.record()
                    dec_events.append((e0, e1))
                else:
                    be.forward(q, k, v, l, batch)

    # ---------------- per-call decode timing for the roofline (eager launches, CUDA events)
    for _ in range(warmup_steps(args)):
        step()
    torch.cuda.synchronize()
    for _ in range(args.steps):
        step(record=True)
    torch.cuda.synchronize()
    dec_ms = [a.elapsed_time(b) for a, b in dec_events]

    # ---------------- device-resident step: the 28 layers as one CUDA graph
    g_dev = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_dev):
        step()
    for _ in range(warmup_steps(args)):
        g_dev.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(args.steps):
        g_dev.replay()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps

    # ---------------- end to end through the public API with host buffers
    host_q = torch.empty(q_all.shape, dtype=torch.bfloat16, pin_memory=True)
    host_q.copy_(q_all.cpu())
    host_kv = torch.empty(kv_all.shape, dtype=torch.bfloat16, pin_memory=True)
    host_kv.copy_(kv_all.cpu())
    host_out = torch.empty((Lyr, B, Hq * D), dtype=torch.bfloat16, pin_memory=True)
    dev_q = torch.empty_like(q_all)
    dev_kv = torch.empty_like(kv_all)
    h2d = torch.cuda.Stream(device=dev)
    d2h = torch.cuda.Stream(device=dev)

    def e2e_layers():
        """Copies and attention of one step; captured once as a CUDA graph.

        Layer l's inputs go host->device on `h2d` and its output device->host
        on `d2h`, so the transfers of other layers overlap the attention of
        layer l (the streams fork from and join the capturing stream).
        """
        comp = torch.cuda.current_stream()
        h2d.wait_stream(comp)
        ready = []
        with torch.cuda.stream(h2d):
            for l in range(Lyr):
                dev_q[l].copy_(host_q[l], non_blocking=True)
                dev_kv[l].copy_(host_kv[l], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
                ready.append(ev)
        d2h.wait_stream(comp)
        with ctx.forward_batch(batch):
            for l in range(Lyr):
                comp.wait_event(ready[l])
                o = layers[l](dev_q[l], dev_kv[l, :, 0], dev_kv[l, :, 1])
                done = torch.cuda.Event()
                done.record(comp)
                d2h.wait_event(done)
                with torch.cuda.stream(d2h):
                    host_out[l].copy_(o, non_blocking=True)
        comp.wait_stream(d2h)
        comp.wait_stream(h2d)

    for _ in range(2):
        e2e_layers()
    torch.cuda.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e):
        e2e_layers()
    meta = batch.attn_metadata
    meta_bytes = 4 * (meta.kv_indptr.numel() + meta.kv_indices.numel() + meta.kv_last_page_len.numel()
                      + meta.cta_indptr.numel() + meta.segs.numel() + meta.merge_indptr.numel())
    req_rows = np.array([r.table_idx for r in reqs])
    req_lens = np.array([r.device_len for r in reqs])

    def e2e_step():
        # prepare_metadata for this step (host numpy + plan + one pinned H2D copy into the
        # graph's metadata buffers), then the captured copies + 28 attention layers
        be.refresh_decode_metadata(meta, req_rows, req_lens)
        g_e2e.replay()

    for _ in range(warmup_steps(args)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    # ---------------- reduce over ranks (max time, summed work)
    dbytes = decode_bytes(pb.lens, P, Hq, Hkv, D, 2)
    sbytes = rope_store_bytes(B, Hq, Hkv, D, 2)
    step_bytes = Lyr * (dbytes + sbytes)
    stats = torch.tensor([ms, e2e_ms, float(np.mean(dec_ms))], dtype=torch.float64, device=dev)
    work = torch.tensor([float(step_bytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(work, op=dist.ReduceOp.SUM)
    ms, e2e_ms, dec_avg = stats.tolist()
    total_bytes = float(work.item())
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9

    peak, peak_kind = measured_peaks()
    achieved = dbytes / (dec_avg * 1e-3) / 1e9
    traffic, traffic_src = decode_traffic()
    launches_per_step = Lyr * 2  # fused RoPE + store, decode (split requests merge inside the decode launch)

    # free the config-2 pools and graphs before the long-context measurement
    del g_dev, g_e2e, kv, be, ctx, layers, q_all, kv_all, dev_q, dev_kv
    set_global_ctx(None)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    ext = None if args.no_extend else measure_extend(dev, args.seed + 31 * rank, args.steps, args.warmup)
    ext1 = None if args.no_extend else measure_extend(dev, args.seed + 31 * rank, args.steps, args.warmup, page_size=1)
    if ext1 is not None:
        ea = measure_extend(dev, args.seed + 31 * rank, args.steps, args.warmup, page_size=1, allocator_order=True)
        ext1["allocator_order"] = {k: ea[k] for k in ("value", "ms_per_call", "roofline", "clocks")}
        ext1["allocator_order"]["packed_group_share"] = ea["config"]["packed_group_share"]
    dec1 = None if args.no_page1 else measure_decode_page1(dev, args.seed + 31 * rank, args.steps, args.warmup)
    c5 = None if args.no_config5 else measure_config5(dev, rank, world, args.seed, args.steps, args.c5_requests)
    e2e4 = None if args.no_config4 else measure_e2e_offline(dev, rank, world, args.seed, n_requests=args.c4_requests,
                                                            fused_proj=not args.no_fused_proj)
    e2e4s = (None if args.no_config4 or args.no_config4_shared else
             measure_e2e_offline(dev, rank, world, args.seed, shared=True, n_requests=args.c4_requests))

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            sub = W.config2_batch(seed=args.seed)
            gbs, per_call, cores = cpu_sample(sub.lens, sub.page_table, P, Hq, Hkv, D, N, 3, 1, args.seed)
            cpu = {"value": round(gbs, 3), "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"1 layer of config 2 (B={B}, sum L={int(sub.lens.sum())}), mean of 3 calls, "
                             f"torch CPU naive gather+mask+SDPA; MLX CPU unavailable on this box"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": warmup_steps(args), "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config2_config(W, world, B, int(pb.lens.sum()), Lyr),
            "roofline": {
                "bound": "hbm", "kernel": "decode_kernel (one b2a_decode call; split requests merged in-launch)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "bytes_per_launch": dbytes, "avg_launch_ms": round(dec_avg, 5),
                # dram__bytes_read.sum + dram__bytes_write.sum of one decode_kernel launch from the
                # committed ncu summary, used only if it was captured on the decode sources timed here
                "traffic": traffic if args.seed == 0 else None,
                "traffic_source": traffic_src if args.seed == 0 else "ncu capture is of seed 0 only",
            },
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                    "h2d_bytes_per_step": int((host_q.numel() + host_kv.numel()) * 2 + meta_bytes),
                    "d2h_bytes_per_step": int(host_out.numel() * 2), "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if ext is not None:
            line["extend_config3"] = ext
        if ext1 is not None:
            line["extend_config3_p1"] = ext1
        if dec1 is not None:
            line["decode_config2_p1"] = dec1
        if c5 is not None:
            line["decode_config5"] = c5
        if e2e4 is not None:
            line["e2e_offline_config4"] = e2e4
        if e2e4s is not None:
            line["e2e_offline_config4_shared"] = e2e4s
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def graph_time_ms(fn, reps: int) -> float:
    """Device time of one call of fn: reps calls captured in one CUDA graph, CUDA events around
    replays, the median over 5 replays divided by reps."""
    import torch

    fn()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        for _ in range(reps):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return float(np.median(times)) / reps


def proj_sweep(rows_list):
    """The decode-step projections of the engine harness's model over its 28 layers.

    Per layer: RMSNorm + qkv_proj, o_proj + residual, RMSNorm + gate_up_proj + SwiGLU,
    down_proj + residual (models/transformer.py:80-82), either as four b2a_proj launches or as
    cuBLAS GEMMs with the residual adds folded in (addmm) plus b2a_rmsnorm and b2a_swiglu.
    Random weights; 28 x 30 MB of weights > L2. One JSON line per token count.
    """
    import torch
    import torch.nn.functional as F

    from minisgl_b200.engine.model import PROJ_PLAIN, PROJ_RESIDUAL, PROJ_SWIGLU, proj, rms_norm, swiglu

    dev = torch.device("cuda", 0)
    Lyr, H, I, QKV, O = 28, 1024, 3072, 4096, 2048
    gen = torch.Generator(device=dev).manual_seed(0)

    def w(o, i):
        return (torch.randn((o, i), device=dev, generator=gen) * 0.02).to(torch.bfloat16)

    layers = [dict(qkv=w(QKV, H), o=w(H, O), gu=w(2 * I, H), d=w(H, I)) for _ in range(Lyr)]
    ones = torch.ones(H, device=dev, dtype=torch.bfloat16)
    wbytes = sum(x.numel() * 2 for lw in layers for x in lw.values())
    peak, kind = measured_peaks()
    for M in rows_list:
        h = torch.randn((M, H), device=dev, generator=gen).to(torch.bfloat16)
        attn = torch.randn((M, O), device=dev, generator=gen).to(torch.bfloat16)

        def fused():
            for lw in layers:
                proj(h, lw["qkv"], PROJ_PLAIN, ones, 1e-6)
                proj(attn, lw["o"], PROJ_RESIDUAL, res=h, out=h)
                proj(proj(h, lw["gu"], PROJ_SWIGLU, ones, 1e-6), lw["d"], PROJ_RESIDUAL, res=h, out=h)

        def unfused():
            x = h
            for lw in layers:
                F.linear(rms_norm(x, ones, 1e-6), lw["qkv"])
                x = torch.addmm(x, attn, lw["o"].t())
                x = torch.addmm(x, swiglu(F.linear(rms_norm(x, ones, 1e-6), lw["gu"])), lw["d"].t())

        line = {"metric": "engine projections, 28 layers of Qwen3-0.6B (us per layer, CUDA graph)", "rows": M,
                "weight_bytes_per_layer": wbytes // Lyr, "hbm_us_per_layer": round(wbytes / Lyr / (peak * 1e3), 2)}
        for name, fn in (("fused", fused), ("unfused", unfused)):
            ms = graph_time_ms(fn, 3)
            line[name] = {"us_per_layer": round(ms * 1e3 / Lyr, 2), "weight_gbs": round(wbytes / (ms * 1e-3) / 1e9, 1)}
        print(json.dumps(line), flush=True)


def decode_sweep(batches):
    """One decode call (config-2 shapes: 16q/8kv/128, bf16, page 16, L~U[100,2048]) per batch
    size, replayed 20 at a time in a CUDA graph. One JSON line per batch size."""
    import torch

    from minisgl_b200 import MHAKVCache
    from minisgl_b200 import workloads as W
    from minisgl_b200.attention import B200AttnBackend
    from minisgl_b200.config import qwen3_0_6b

    dev = torch.device("cuda", 0)
    cfg = qwen3_0_6b()
    N = W.CONFIG2["num_slots"]
    kv = MHAKVCache(1, N, 8, 128, torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(0)
    kv.k[0].normal_(generator=gen)
    kv.v[0].normal_(generator=gen)
    peak, kind = measured_peaks()
    for B in batches:
        pb = W.config2_batch(seed=1, batch=B)
        be = B200AttnBackend(cfg, kv, pb.page_table, page_size=16)
        meta = be.decode_metadata_from_lens(pb.rows, pb.lens)
        q = torch.randn((B, 16, 128), device=dev, generator=gen).to(torch.bfloat16)
        ms = graph_time_ms(lambda: be.forward_decode(q, 0, meta), 20)
        nbytes = decode_bytes(pb.lens, 16, 16, 8, 128, 2)
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"metric": "decode call, config-2 shapes (CUDA graph)", "batch": B,
                          "sum_ctx_tokens": int(pb.lens.sum()), "bytes_per_call": nbytes, "us_per_call": round(ms * 1e3, 2),
                          "gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "peak_kind": kind}), flush=True)


def main():
    args = parse_args()
    if args.proj_sweep:
        proj_sweep([int(x) for x in args.proj_sweep.split(",")])
    elif args.decode_sweep:
        decode_sweep([int(x) for x in args.decode_sweep.split(",")])
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
