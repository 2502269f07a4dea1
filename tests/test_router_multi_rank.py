"""Prefix-cache hits survive request partitioning (the prefix-affinity router), on CPU ranks.

Workload: config 4 with shared prefixes (workloads.config4_shared_workload: 16
system prompts of 512-2048 tokens, each starting 16 of the 256 requests). Every
rank runs the engine's host scheduler (engine.scheduler.HostScheduler: admission,
chunked prefill, paging, the radix prefix cache of kvcache/radix_cache.py and
the processing of sampled tokens) over its share of the requests, with a stand-in
for the model's sampled tokens (nothing here depends on token values: ignore_eos,
and outputs never prefix another prompt). The ranks are gloo processes; the
job's prefix-hit tokens are summed with all_reduce.

* with the router (route_requests: first-page groups kept on one rank) the hit
  total at 2 and 4 ranks stays within 5 % of one rank's;
* partitioning the same requests without regard to prefixes (longest-first
  sharding) loses a large part of them, which is what the router is for.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def run_host_only(prompts, outs, cfg) -> dict:
    """LLM.generate's loop (feed about one prefill budget of prompts at a time, prefill first,
    else one decode step) on the host scheduler alone; returns its counters."""
    from minisgl_b200.core import SamplingParams
    from minisgl_b200.engine import HostScheduler

    P = cfg.page_size
    max_seq_len = cfg.max_seq_len or cfg.num_tokens
    page_table = np.zeros((cfg.max_running_req + 1, max_seq_len), dtype=np.int32)
    hs = HostScheduler(cfg, page_table, cfg.num_tokens // P - 1)
    queue = [(i, np.asarray(p, np.int32), SamplingParams(max_tokens=int(n), ignore_eos=True))
             for i, (p, n) in enumerate(zip(prompts, outs))]
    produced = {i: 0 for i in range(len(prompts))}

    hs.on_token = lambda req, tok, fin: produced.__setitem__(req.uid, produced[req.uid] + 1)
    while True:
        budget = 0
        while queue and budget < cfg.max_extend_tokens:
            uid, ids, sp = queue.pop(0)
            budget += len(ids)
            hs.prefill.add_one_req(uid, ids, sp)
        if hs.idle and not queue:
            break
        batch = hs.next_batch()
        assert batch is not None, "a pending request can never fit"
        for r in batch.reqs:
            r.complete_one()
        hs.decode.filter_reqs(batch.reqs)
        hs.process_tokens(batch, [(r.uid * 7919 + r.device_len) % 10000 for r in batch.reqs])
    hs.cache.check_integrity()
    assert [produced[i] for i in range(len(prompts))] == [int(n) for n in outs]
    return {"hits": hs.num_prefix_hit_tokens, "prefill": hs.num_prefill_tokens, "outputs": hs.num_output_tokens}


def _cfg():
    from minisgl_b200 import workloads as W
    from minisgl_b200.engine import EngineConfig, qwen3_0_6b_spec

    c = W.CONFIG4_SHARED
    return EngineConfig(spec=qwen3_0_6b_spec(), max_running_req=c["max_running_req"], page_size=c["page_size"],
                        num_tokens=c["num_tokens"], max_extend_tokens=c["max_extend_tokens"])


def _rank_main(rank: int, world: int, port: int, policy: str, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from minisgl_b200 import workloads as W
        from minisgl_b200.engine.router import route_requests

        prompts, outs, _ = W.config4_shared_workload(seed=0)
        cost = np.array([len(p) for p in prompts]) + outs
        if policy == "router":
            mine = route_requests(prompts, cost, world, page_size=W.CONFIG4_SHARED["page_size"])[rank]
        else:
            mine = W.shard_requests(cost, world)[rank]
        res = run_host_only([prompts[i] for i in mine], outs[mine], _cfg())
        t = torch.tensor([res["hits"], res["prefill"], res["outputs"]], dtype=torch.int64)
        dist.all_reduce(t)
        if rank == 0:
            out_q.put(t.tolist())
    finally:
        dist.destroy_process_group()


def _job(world: int, policy: str):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, policy, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    return q.get(timeout=10)


def test_host_scheduler_single_rank_hits_the_shared_prefixes():
    from minisgl_b200 import workloads as W

    prompts, outs, group = W.config4_shared_workload(seed=0)
    res = run_host_only(prompts, outs, _cfg())
    # each group's system prompt is computed about once and then served from the cache: at
    # least 12 of the 16 requests of every group hit at least its page-aligned system prompt
    sys_len = _system_lengths(prompts, group)
    assert res["hits"] >= sum(12 * (n // 16 * 16) for n in sys_len), (res, sys_len)
    assert res["outputs"] == int(outs.sum())


def _system_lengths(prompts, group):
    """Length of each group's shared system prompt (the common prefix of its prompts)."""
    lens = []
    for g in sorted(set(group.tolist())):
        members = [prompts[i] for i in np.nonzero(group == g)[0]]
        n = min(len(p) for p in members)
        first = members[0]
        for p in members[1:]:
            n = min(n, int(np.argmin(np.append(p[:n] == first[:n], False))))
        lens.append(n)
    return lens


@pytest.mark.parametrize("world", [2, 4])
def test_router_keeps_prefix_hits_across_ranks(world):
    from minisgl_b200 import workloads as W

    prompts, outs, group = W.config4_shared_workload(seed=0)
    one = run_host_only(prompts, outs, _cfg())
    routed = _job(world, "router")
    assert routed[2] == int(outs.sum())  # every request ran exactly once across the ranks
    assert routed[0] >= 0.98 * one["hits"], (routed, one)
    # without prefix affinity a group's system prompt is computed again on most ranks
    blind = _job(world, "lpt")
    sys_pages = sum(n // 16 * 16 for n in _system_lengths(prompts, group))
    assert blind[0] <= routed[0] - 0.5 * (world - 1) * sys_pages, (blind, routed, sys_pages)
