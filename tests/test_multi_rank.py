"""Request-partitioned multi-rank logic on CPU (gloo, world_size 2).

The attention path shards by request with no data-path collective. These
tests check the host-side sharding every rank computes independently (all
ranks agree, the shards are disjoint and cover the batch) and the only
collectives the bench uses: a barrier and the max-over-ranks timing
reduction plus a summed byte count.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank: int, world: int, port: int, out):
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "mini-sglang-mlx_b200")]
    import torch
    import torch.distributed as dist

    from minisgl_b200 import workloads as W

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = W.config5_lens(seed=0, batch=97)
        shards = W.shard_requests(lens, world)
        mine = shards[rank]
        # every rank computed the same partition independently
        gathered = [None] * world
        dist.all_gather_object(gathered, [s.tolist() for s in shards])
        same = all(g == gathered[0] for g in gathered)
        # bench-style reduction: max time, summed work
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        w = torch.tensor([float(lens[mine].sum())], dtype=torch.float64)
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(w, op=dist.ReduceOp.SUM)
        out[rank] = (same, mine.tolist(), float(t.item()), float(w.item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharding_and_reductions_gloo(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from minisgl_b200 import workloads as W

    lens = W.config5_lens(seed=0, batch=97)
    res = [out[r] for r in range(world)]
    assert all(r[0] for r in res)
    ids = sorted(i for r in res for i in r[1])
    assert ids == list(range(97))
    assert all(r[2] == float(world) for r in res)  # max over ranks
    assert all(r[3] == float(lens.sum()) for r in res)  # total work
    loads = [lens[r[1]].sum() for r in res]
    assert max(loads) - min(loads) <= lens.max()
