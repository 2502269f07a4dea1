"""Multi-GPU request router with prefix affinity.

Every GPU runs its own engine with its own radix prefix cache, so a cached
prefix only helps the requests routed to the GPU that holds it. Requests
whose prompts share their first page of tokens (the radix tree's first-level
key, kvcache/radix_cache.py:247-268) are therefore kept on one rank. Groups
of such requests are placed longest-processing-time first on the least
loaded rank (load = prompt + output tokens); a group bigger than one rank's
fair share is cut into consecutive chunks, so balance never depends on how
the prompts cluster. Deterministic for a given input.
"""

from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np


def prefix_key(ids: np.ndarray, page_size: int) -> bytes:
    """First-page key of a prompt; prompts shorter than a page key on all their tokens."""
    ids = np.asarray(ids, dtype=np.int32)
    return ids[: max(page_size, 1)].tobytes()


def route_requests(prompts: Sequence[np.ndarray], costs: np.ndarray, world: int,
                   page_size: int = 16) -> List[np.ndarray]:
    """Request ids of each rank (sorted ascending)."""
    costs = np.asarray(costs, dtype=np.float64)
    n = len(prompts)
    if world <= 1:
        return [np.arange(n, dtype=np.int64)]
    groups: Dict[bytes, List[int]] = {}
    for i, p in enumerate(prompts):
        groups.setdefault(prefix_key(p, page_size), []).append(i)
    share = costs.sum() / world
    units: List[List[int]] = []
    for members in groups.values():
        members = sorted(members)
        total = costs[members].sum()
        if total <= share or len(members) == 1:
            units.append(members)
            continue
        # cut an oversized group into chunks of about one share each
        chunk: List[int] = []
        acc = 0.0
        for i in members:
            chunk.append(i)
            acc += costs[i]
            if acc >= share:
                units.append(chunk)
                chunk, acc = [], 0.0
        if chunk:
            units.append(chunk)
    units.sort(key=lambda u: (-costs[u].sum(), u[0]))
    load = np.zeros(world)
    ranks: List[List[int]] = [[] for _ in range(world)]
    for u in units:
        r = int(np.argmin(load))
        ranks[r].extend(u)
        load[r] += costs[u].sum()
    return [np.array(sorted(r), dtype=np.int64) for r in ranks]
