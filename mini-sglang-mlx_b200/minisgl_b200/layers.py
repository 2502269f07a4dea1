"""Rotary embedding and AttentionLayer (reference python/minisgl_mlx/layers.py).

``AttentionLayer.__call__`` keeps the reference order (layers.py:103-111):
rotate q and k, store the rotated k and v into the pool at ``batch.out_loc``,
run the backend, reshape to ``[T, Hq * D]``. Here the first three steps are ONE
kernel (b2a_rope_store) that rotates q and k in place and scatters k and v, so
the stored k is bit-identical to the k the backend sees.

Inverse frequencies (reference layers.py:31-43,59-74 and mx.fast.rope's
definition inv_freq_i = base^(-2i/dims), or 1/freqs[i] for llama3) are
computed once on the host: base^(-2i/dims) in float64 rounded to float32,
the llama3 periods in float32 in the reference's own operation order (their
reciprocal is one correctly rounded float32 division); the kernel uses
angle = fl32(fl32(pos * scale) * inv_freq[i]) with an accurate sincos.
"""

from __future__ import annotations

import math
from typing import Any, Dict

import numpy as np
import torch

from . import _native as nat
from .config import RotaryConfig
from .core import get_global_ctx
from .kvcache.pool import current_stream_ptr, dtype_code


def llama3_freqs(dims: int, base: float, scaling: Dict[str, Any]) -> np.ndarray:
    """Wavelength-scaled rotary periods of Llama 3 (reference layers.py:59-74), float32.

    The reference evaluates this on MLX float32 arrays; the same operations in the same
    order on numpy float32 arrays (Python scalars never widen them) give the same table.
    """
    factor = scaling["factor"]
    low = scaling.get("low_freq_factor", 1.0)
    high = scaling.get("high_freq_factor", 4.0)
    old_ctx = scaling.get("original_max_position_embeddings", 8192)
    low_wavelen = old_ctx / low
    high_wavelen = old_ctx / high
    freqs = base ** (np.arange(0, dims, 2, dtype=np.float32) / dims)
    wavelens = 2 * math.pi * freqs
    freqs = np.where(wavelens > low_wavelen, freqs * factor, freqs)
    is_medium = (wavelens > high_wavelen) & (wavelens < low_wavelen)
    smooth = (old_ctx / wavelens - low) / (high - low)
    smooth_freqs = freqs / ((1 - smooth) / factor + smooth)
    return np.where(is_medium, smooth_freqs, freqs)


def rope_tables(config: RotaryConfig) -> tuple[np.ndarray, float]:
    """(inv_freq float32 [rotary_dim/2], position scale) for a rotary config."""
    dims = config.rotary_dim
    scale = 1.0
    scaling = config.scaling
    rope_type = "default"
    if scaling:
        rope_type = scaling.get("rope_type", scaling.get("type", "default"))
    if rope_type == "llama3":
        inv = 1.0 / llama3_freqs(dims, config.base, scaling)
    elif rope_type in ("default", "linear"):
        inv = float(config.base) ** (-np.arange(0, dims, 2, dtype=np.float64) / dims)
        if rope_type == "linear":
            scale = 1.0 / scaling["factor"]
    else:
        raise NotImplementedError(f"rope_scaling type {rope_type!r} is not supported yet")
    return inv.astype(np.float32), scale


class RotaryEmbedding:
    """rotate-half RoPE (mx.fast.rope, traditional=False) on the GPU."""

    def __init__(self, config: RotaryConfig, device: torch.device | None = None) -> None:
        inv, scale = rope_tables(config)
        self.dims = config.rotary_dim
        self.scale = scale
        self.inv_freq_host = inv
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.inv_freq = torch.from_numpy(inv).to(dev)

    def __call__(self, x: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """Return a rotated copy of x ``[T, H, D]`` (reference layers.py:45-56)."""
        y = x.contiguous().clone()
        T, H, D = y.shape
        nat.call(
            "b2a_rope_store", None, 0, y.data_ptr(), y.stride(0), None, 0, positions.data_ptr(), None,
            None, None, 0, self.inv_freq.data_ptr(), float(self.scale), self.dims, T, 0, H, D,
            dtype_code(y.dtype), current_stream_ptr(y.device),
        )
        return y

    def rope_store_(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
                    out_loc: torch.Tensor, kv_cache, layer_id: int, q_norm_w: torch.Tensor | None = None,
                    k_norm_w: torch.Tensor | None = None, eps: float = 1e-6,
                    q_out: torch.Tensor | None = None) -> None:
        """Rotate q, k IN PLACE and scatter rotated k and v into ``kv_cache`` layer ``layer_id``.

        With ``q_norm_w`` / ``k_norm_w`` the per-head RMSNorm (Qwen3) is applied first,
        in the same kernel (b2a_qknorm_rope_store). With ``q_out`` ([T, Hq, D],
        contiguous) the final q rows go there and q's rows are used as scratch.
        """
        T, Hq, D = q.shape
        Hkv = k.shape[1]
        for name, t in (("q", q), ("k", k), ("v", v)):
            assert t.stride(2) == 1 and t.stride(1) == D, f"{name} rows must be [H, D] contiguous"
        assert positions.dtype == torch.int32 and out_loc.dtype == torch.int32
        for w in (q_norm_w, k_norm_w):
            assert w is None or (w.shape == (D,) and w.dtype == q.dtype and w.is_contiguous())
        assert q_out is None or (q_out.shape == q.shape and q_out.is_contiguous() and q_out.dtype == q.dtype)
        nat.call(
            "b2a_qknorm_rope_store", q.data_ptr(), q.stride(0), None if q_out is None else q_out.data_ptr(),
            k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
            None if q_norm_w is None else q_norm_w.data_ptr(), None if k_norm_w is None else k_norm_w.data_ptr(),
            float(eps), positions.data_ptr(), out_loc.data_ptr(), kv_cache.k_cache(layer_id).data_ptr(),
            kv_cache.v_cache(layer_id).data_ptr(), kv_cache.num_tokens, self.inv_freq.data_ptr(),
            float(self.scale), self.dims, T, Hq, Hkv, D, dtype_code(q.dtype), current_stream_ptr(q.device),
        )


class AttentionLayer:
    """reference layers.py:77-111; parameter-free, reads the global Context."""

    def __init__(self, layer_id: int, num_qo_heads: int, num_kv_heads: int, head_dim: int,
                 rotary_config: RotaryConfig) -> None:
        assert num_qo_heads % num_kv_heads == 0
        self.layer_id = layer_id
        self.num_qo_heads = num_qo_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.rotary = RotaryEmbedding(rotary_config)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm_w: torch.Tensor | None = None,
                 k_norm_w: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
        """q ``[T, Hq, D]``, k/v ``[T, Hkv, D]`` -> o ``[T, Hq * D]``. q and k are rotated in place.

        Extension for Qwen3-style models: with ``q_norm_w`` / ``k_norm_w`` the per-head
        RMSNorm that the model would apply before this call (models/transformer.py:54-56)
        is fused into the RoPE + store kernel; q may then be a strided view (e.g. of a
        fused qkv projection) and the rotated q goes to a fresh contiguous tensor.
        """
        ctx = get_global_ctx()
        batch = ctx.batch
        fused = q_norm_w is not None or k_norm_w is not None
        if fused or not q.is_contiguous():
            q_out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
            self.rotary.rope_store_(q, k, v, batch.positions, batch.out_loc, ctx.kv_cache, self.layer_id,
                                    q_norm_w, k_norm_w, eps, q_out=q_out)
            q = q_out
        else:
            self.rotary.rope_store_(q, k, v, batch.positions, batch.out_loc, ctx.kv_cache, self.layer_id)
        o = ctx.attn_backend.forward(q, k, v, self.layer_id, batch)
        return o.reshape(o.shape[0], self.num_qo_heads * self.head_dim)
