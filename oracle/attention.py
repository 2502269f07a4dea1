"""CPU oracle of the reference attention path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker / the timed CPU baseline. The
product (minisgl_b200) never calls it.

It restates, in numpy float64 by default, the arithmetic of the reference's
naive backend and the surrounding hot path (paths are inside the reference
project):

  align_up                  python/minisgl_mlx/utils.py:37-46
  naive_prepare_decode      python/minisgl_mlx/attention/naive.py:36-48
  naive_forward_decode      python/minisgl_mlx/attention/naive.py:50-60
  metal_prepare_decode      python/minisgl_mlx/attention/metal.py:145-152
  prepare_prefill           python/minisgl_mlx/attention/base.py:70-83
  forward_prefill           python/minisgl_mlx/attention/base.py:85-105
  forward_prefill_torch     the same, pool branch, torch BLAS on the CPU (benchmark-sized batches)
  rope                      python/minisgl_mlx/layers.py:45-56 (mx.fast.rope, traditional=False)
  store_kv                  python/minisgl_mlx/kvcache/pool.py:47-50
  attention_layer           python/minisgl_mlx/layers.py:103-111
  sdpa                      mx.fast.scaled_dot_product_attention semantics as the
                            reference calls it (attention/base.py:97-103,
                            attention/naive.py:53-59): softmax(scale q k^T + mask) v,
                            GQA by head grouping, boolean mask True = keep,
                            mask="causal" aligned to the bottom-right corner.

The arithmetic of SDPA and RoPE lives in the third-party `mlx` package
(declared as mlx>=0.29 in pyproject.toml:13, no lockfile, so the version is
unpinned) which cannot be imported here. The restatement follows the
published definitions; the reference's own test (tests/test_attention.py)
holds no golden vectors. Parity of this oracle is pinned by known-answer
tests and by running the reference's own Metal kernel body on the CPU
(oracle/metal_ref), see tests/test_oracle.py.

bf16 values are carried as float32 arrays holding bf16-representable values
(``bf16_round`` is round-to-nearest-even on the float32 bit pattern).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np


# --------------------------------------------------------------------------- numerics
def align_up(a: int, b: int) -> int:
    return (a + b - 1) // b * b


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    nan = np.isnan(x)
    out = r.astype(np.uint32).view(np.float32)
    out = np.where(nan, np.float32(np.nan), out)
    return out.astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "bfloat16":
        return bf16_round(np.asarray(x, dtype=np.float32))
    if dtype == "float16":
        return np.asarray(x, dtype=np.float16).astype(np.float32)
    raise ValueError(dtype)


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, mask: Optional[np.ndarray] = None,
         causal: bool = False, acc=np.float64) -> np.ndarray:
    """softmax(scale * q k^T [+ mask]) v.

    q [B, Hq, Lq, D], k/v [B, Hkv, Lkv, D]; query head h reads kv head h // (Hq / Hkv).
    mask: bool, broadcast to [B, Hq, Lq, Lkv], True = attend. causal: query i attends
    keys j <= i + (Lkv - Lq).
    """
    B, Hq, Lq, D = q.shape
    Hkv, Lkv = k.shape[1], k.shape[2]
    G = Hq // Hkv
    qf = q.astype(acc)
    kf = np.repeat(k.astype(acc), G, axis=1)
    vf = np.repeat(v.astype(acc), G, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", qf, kf) * acc(scale)
    keep = np.ones((B, Hq, Lq, Lkv), dtype=bool)
    if mask is not None:
        keep &= np.broadcast_to(mask, keep.shape)
    if causal:
        off = Lkv - Lq
        keep &= (np.arange(Lkv)[None, :] <= np.arange(Lq)[:, None] + off)[None, None]
    s = np.where(keep, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p = np.where(keep, p, 0.0)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, vf)


# --------------------------------------------------------------------------- decode
def naive_prepare_decode(page_table: np.ndarray, rows: Sequence[int], lens: Sequence[int]):
    """attention/naive.py:36-48: padded indices to align_up(max, 128) (capped) and a bool mask."""
    lens = np.asarray(lens)
    rows = np.asarray(rows)
    max_len = min(align_up(int(lens.max()), 128), page_table.shape[1])
    kv_indices = page_table[rows, :max_len]
    mask = np.arange(max_len)[None, :] < lens[:, None]
    return kv_indices, mask[:, None, None, :]


def naive_forward_decode(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, kv_indices: np.ndarray,
                         mask: np.ndarray, scale: float, acc=np.float64) -> np.ndarray:
    """attention/naive.py:50-60: gather [B, L, Hkv, D] -> [B, Hkv, L, D], masked SDPA. q [B, Hq, D]."""
    k = k_pool[kv_indices].transpose(0, 2, 1, 3)
    v = v_pool[kv_indices].transpose(0, 2, 1, 3)
    o = sdpa(q[:, :, None, :], k, v, scale, mask=mask, acc=acc)
    return o[:, :, 0, :]


def metal_prepare_decode(page_table: np.ndarray, rows: Sequence[int], lens: Sequence[int]):
    """attention/metal.py:145-152: token CSR (kv_indptr [B+1], kv_indices = row-major valid entries)."""
    lens = np.asarray(lens)
    rows = np.asarray(rows)
    max_len = int(lens.max())
    valid = np.arange(max_len)[None, :] < lens[:, None]
    kv_indices = page_table[rows, :max_len][valid]
    kv_indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return kv_indptr, kv_indices.astype(np.int32)


def reference_decode_per_request(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray,
                                 indices_per_req: List[np.ndarray], scale: float) -> np.ndarray:
    """tests/test_attention.py:10-16: per-request contiguous gather + unmasked SDPA."""
    outs = []
    for b, idx in enumerate(indices_per_req):
        k = k_pool[np.asarray(idx)].transpose(1, 0, 2)[None]
        v = v_pool[np.asarray(idx)].transpose(1, 0, 2)[None]
        outs.append(sdpa(q[b:b + 1, :, None], k, v, scale)[:, :, 0])
    return np.concatenate(outs)


# --------------------------------------------------------------------------- prefill
@dataclass
class PrefillMeta:
    last_indices: np.ndarray
    q_offsets: List[int]
    kv_indices: List[Optional[np.ndarray]]


def prepare_prefill(page_table: np.ndarray, table_idx: Sequence[int], cached_len: Sequence[int],
                    device_len: Sequence[int]) -> PrefillMeta:
    """attention/base.py:70-83."""
    extend = [d - c for c, d in zip(cached_len, device_len)]
    q_offsets = np.concatenate([[0], np.cumsum(extend)]).astype(np.int64).tolist()
    kv_indices: List[Optional[np.ndarray]] = []
    for row, c, d in zip(table_idx, cached_len, device_len):
        kv_indices.append(None if c == 0 else page_table[row, :d].copy())
    last = np.array(q_offsets[1:], dtype=np.int32) - 1
    return PrefillMeta(last_indices=last, q_offsets=q_offsets, kv_indices=kv_indices)


def forward_prefill(q: np.ndarray, k: np.ndarray, v: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray,
                    meta: PrefillMeta, scale: float, acc=np.float64) -> np.ndarray:
    """attention/base.py:85-105: one SDPA per request, causal (bottom-right) when Lq > 1."""
    outs = []
    for i, kv_idx in enumerate(meta.kv_indices):
        s, e = meta.q_offsets[i], meta.q_offsets[i + 1]
        qi = q[s:e]
        if kv_idx is None:
            ki, vi = k[s:e], v[s:e]
        else:
            ki, vi = k_pool[kv_idx], v_pool[kv_idx]
        oi = sdpa(qi.transpose(1, 0, 2)[None], ki.transpose(1, 0, 2)[None], vi.transpose(1, 0, 2)[None],
                  scale, causal=(e - s) > 1, acc=acc)
        outs.append(oi[0].transpose(1, 0, 2))
    return outs[0] if len(outs) == 1 else np.concatenate(outs, axis=0)


def forward_prefill_torch(q, k_pool, v_pool, q_offsets: Sequence[int], kv_indices: List[np.ndarray], scale: float,
                          dtype=None):
    """attention/base.py:85-105 with every request reading its keys from the pool, in torch on the CPU.

    The same arithmetic as ``forward_prefill`` (per-request SDPA, bottom-right causal when
    Lq > 1, GQA by head grouping), written with BLAS matmuls so that batches of the
    benchmark's size (thousands of query rows over thousands of keys) finish in seconds.
    q [T, Hq, D], pools [N, Hkv, D] (torch CPU tensors, any float dtype); the math runs in
    ``dtype`` (default float64). Returns [T, Hq, D] in ``dtype``.
    """
    import torch

    dtype = dtype or torch.float64
    T, Hq, D = q.shape
    Hkv = k_pool.shape[1]
    G = Hq // Hkv
    out = torch.empty((T, Hq, D), dtype=dtype)
    for i, idx in enumerate(kv_indices):
        s0, s1 = int(q_offsets[i]), int(q_offsets[i + 1])
        Lq = s1 - s0
        if Lq == 0:
            continue
        sel = torch.from_numpy(np.asarray(idx, dtype=np.int64))
        kr = k_pool[sel].to(dtype).permute(1, 0, 2)  # [Hkv, Lkv, D]
        vr = v_pool[sel].to(dtype).permute(1, 0, 2)
        Lkv = kr.shape[1]
        qr = q[s0:s1].to(dtype).reshape(Lq, Hkv, G, D).permute(1, 2, 0, 3).reshape(Hkv, G * Lq, D)
        sc = torch.matmul(qr, kr.transpose(1, 2)) * scale  # [Hkv, G*Lq, Lkv]
        if Lq > 1:
            row = torch.arange(Lq).repeat(G)  # query row of each (g, i) line
            keep = torch.arange(Lkv)[None, :] <= (row[:, None] + (Lkv - Lq))
            sc.masked_fill_(~keep[None], float("-inf"))
        p = torch.softmax(sc, dim=-1)
        o = torch.matmul(p, vr)  # [Hkv, G*Lq, D]
        out[s0:s1] = o.reshape(Hkv, G, Lq, D).permute(2, 0, 1, 3).reshape(Lq, Hq, D)
    return out


# --------------------------------------------------------------------------- rope + store
def rope_inv_freq(dims: int, base: float) -> np.ndarray:
    """base^(-2i/dims), i < dims/2, computed in float64 and rounded to float32."""
    return (float(base) ** (-np.arange(0, dims, 2, dtype=np.float64) / dims)).astype(np.float32)


def rope(x: np.ndarray, positions: np.ndarray, dims: int, inv_freq: np.ndarray, scale: float = 1.0,
         out_dtype: str = "float32") -> np.ndarray:
    """mx.fast.rope(x[T,H,1,D], dims, traditional=False, offset=positions) as layers.py:45-56 calls it.

    angle = fl32(fl32(pos * scale) * inv_freq[i]); features (i, i + dims/2) for i < dims/2 are
    rotated, features >= dims pass through. Rotation in float64, result rounded to out_dtype.
    """
    x = np.asarray(x, dtype=np.float64)
    half = dims // 2
    pos32 = (positions.astype(np.float32) * np.float32(scale)).astype(np.float32)
    ang = (pos32[:, None] * inv_freq.astype(np.float32)[None, :]).astype(np.float32).astype(np.float64)
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    y = x.copy()
    x1, x2 = x[..., :half], x[..., half:dims]
    y[..., :half] = x1 * c - x2 * s
    y[..., half:dims] = x2 * c + x1 * s
    return round_to(y, out_dtype)


def store_kv(k_pool: np.ndarray, v_pool: np.ndarray, k: np.ndarray, v: np.ndarray, out_loc: np.ndarray) -> None:
    """kvcache/pool.py:47-50: k_pool[out_loc] = k, v_pool[out_loc] = v (in place)."""
    k_pool[out_loc] = k
    v_pool[out_loc] = v


def attention_layer_prefill(q, k, v, positions, out_loc, k_pool, v_pool, meta: PrefillMeta, dims, inv_freq,
                            rope_scale, scale, dtype: str):
    """layers.py:103-111 for a prefill batch: rope(q), rope(k), store, forward_prefill."""
    qr = rope(q, positions, dims, inv_freq, rope_scale, dtype)
    kr = rope(k, positions, dims, inv_freq, rope_scale, dtype)
    store_kv(k_pool, v_pool, kr, v, out_loc)
    return forward_prefill(qr, kr, v, k_pool, v_pool, meta, scale), qr, kr
