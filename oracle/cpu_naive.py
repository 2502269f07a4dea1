"""Timed CPU baseline: the reference's naive decode in torch on the host cores.

TEST/BENCH INFRASTRUCTURE ONLY (bench.py's cpu_baseline leg and --impl
reference arm). Restates python/minisgl_mlx/attention/naive.py:36-60 -- pad
the page-table rows to align_up(max len, 128) (capped), gather K/V
[B, L_max, Hkv, D], boolean mask j < len, SDPA -- with torch CPU ops, all host
threads, bf16 storage and fp32 math (the MLX CPU path cannot run here).
"""

from __future__ import annotations

import numpy as np
import torch

from .attention import align_up


def naive_decode_torch(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, page_table: np.ndarray,
                       rows: np.ndarray, lens: np.ndarray, scale: float) -> torch.Tensor:
    """q [B, Hq, D], pools [N, Hkv, D] (CPU tensors) -> o [B, Hq, D] (float32)."""
    lens = np.asarray(lens)
    B, Hq, D = q.shape
    Hkv = k_pool.shape[1]
    max_len = min(align_up(int(lens.max()), 128), page_table.shape[1])
    idx = torch.from_numpy(np.ascontiguousarray(page_table[np.asarray(rows), :max_len])).long()
    mask = torch.arange(max_len)[None, :] < torch.from_numpy(lens)[:, None]
    k = k_pool[idx].transpose(1, 2)  # [B, Hkv, L, D]
    v = v_pool[idx].transpose(1, 2)
    qf = q.float().view(B, Hkv, Hq // Hkv, D)
    s = torch.einsum("bhgd,bhld->bhgl", qf, k.float()) * scale
    s.masked_fill_(~mask[:, None, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhgl,bhld->bhgd", p, v.float())
    return o.reshape(B, Hq, D)
