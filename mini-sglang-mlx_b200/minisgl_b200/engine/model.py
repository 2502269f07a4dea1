"""Random-initialised Qwen3 decoder over packed tokens (the engine harness's model).

Structure of python/minisgl_mlx/models/transformer.py:33-116: per layer an
RMSNorm, a fused q/k/v projection, per-head q/k RMSNorm (Qwen3; fused into
the AttentionLayer's RoPE + KV-store kernel), the AttentionLayer (then the
attention backend), the output
projection, RMSNorm and a fused gate/up SwiGLU MLP, with residuals; a final
RMSNorm and tied embeddings as the LM head. Prefill keeps only each
request's last token before the head (``attn_metadata.last_indices``).

Inputs are packed ``[T]`` token ids. A bf16 step of at most 32 tokens (every
decode step of a rank holding <= 32 requests) runs each layer's projections
as ``b2a_proj`` launches with their neighbours fused: RMSNorm + qkv_proj,
o_proj + residual add (in place), RMSNorm + gate_up_proj + SwiGLU, down_proj
+ residual add -- four launches where the unfused form takes seven. Larger
steps (prefill chunks, big decode batches) and fp32 models use cuBLAS through
``F.linear``, with the two residual adds folded into the o_proj and down GEMMs
(``torch.addmm`` with beta = 1: one rounding instead of two), SwiGLU as one
library kernel (``b2a_swiglu``, as the reference's mx.compile'd ``swiglu`` is
one kernel) and the RMSNorms as ``b2a_rmsnorm``. In prefill the final norm
gathers the last tokens itself (one kernel for the gather and the norm).
Weights are drawn N(0, 0.02) from a seeded generator (there are no
checkpoints on this machine), norms start at 1.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.nn.functional as F

from .. import _native as nat
from ..config import ModelConfig, RotaryConfig
from ..core import get_global_ctx
from ..kvcache.pool import dtype_code
from ..layers import AttentionLayer


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up of a ``[T, 2F]`` gate/up projection in one kernel (b2a_swiglu).

    Reference: python/minisgl_mlx/models/transformer.py:26-30 and :67-69.
    """
    T, F2 = gate_up.shape
    out = torch.empty((T, F2 // 2), dtype=gate_up.dtype, device=gate_up.device)
    nat.call("b2a_swiglu", gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(), T, F2 // 2,
             dtype_code(gate_up.dtype), torch.cuda.current_stream().cuda_stream)
    return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, rows: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of the rows of ``x`` ``[T, H]`` (b2a_rmsnorm), optionally of ``x[rows]`` only.

    Reference: nn.RMSNorm of python/minisgl_mlx/models/transformer.py:77-82; with ``rows``
    the last-token gather plus final norm of :109-113 in one kernel.
    """
    T, H = x.shape
    assert x.stride(1) == 1 and w.dtype == x.dtype
    n = T if rows is None else rows.numel()
    y = torch.empty((n, H), dtype=x.dtype, device=x.device)
    if rows is not None:
        assert rows.dtype == torch.int32 and rows.is_contiguous()
    nat.call("b2a_rmsnorm", x.data_ptr(), x.stride(0), T, 0 if rows is None else rows.data_ptr(), n, w.data_ptr(),
             float(eps), H, y.data_ptr(), dtype_code(x.dtype), torch.cuda.current_stream().cuda_stream)
    return y


PROJ_PLAIN, PROJ_RESIDUAL, PROJ_SWIGLU = 0, 1, 2
PROJ_MAX_ROWS = 64  # token rows of one b2a_proj launch
# steps the model runs through b2a_proj: measured over the 28 layers of Qwen3-0.6B (CUDA
# graph, B200) the fused layer takes 12 / 23 / 36 us at 8 / 32 / 64 rows against 33 / 31 /
# 30 us for cuBLAS + separate norm and SwiGLU kernels (every CTA re-reads all token rows,
# a cost that grows with the rows), so larger steps keep the library GEMMs
FUSED_MAX_ROWS = 32


def proj(x: torch.Tensor, w: torch.Tensor, mode: int, norm_w: torch.Tensor | None = None, eps: float = 0.0,
         res: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``[T, K] x [N, K]^T`` for T <= 64 bf16 rows with the RMSNorm in front (``norm_w``) and
    the residual add (``PROJ_RESIDUAL``, ``out`` may be ``res``) or SwiGLU (``PROJ_SWIGLU``,
    ``[T, N/2]``) behind, in one launch (b2a_proj).

    Reference: python/minisgl_mlx/models/transformer.py:80-82 (DecoderLayer.__call__) with the
    projections of :41-42 and :64-65 and ``swiglu`` of :26-30.
    """
    T, K = x.shape
    N = w.shape[0]
    assert x.stride(1) == 1 and w.is_contiguous() and w.shape[1] == K
    if out is None:
        out = torch.empty((T, N // 2 if mode == PROJ_SWIGLU else N), dtype=x.dtype, device=x.device)
    nat.call("b2a_proj", x.data_ptr(), x.stride(0), T, K, w.data_ptr(), N,
             0 if norm_w is None else norm_w.data_ptr(), float(eps), 0 if res is None else res.data_ptr(),
             0 if res is None else res.stride(0), out.data_ptr(), out.stride(0), mode, dtype_code(x.dtype),
             torch.cuda.current_stream().cuda_stream)
    return out


@dataclass(frozen=True)
class Qwen3Spec:
    attn: ModelConfig  # layers, heads, head_dim, rotary
    hidden_size: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True


def qwen3_0_6b_spec() -> Qwen3Spec:
    """Qwen3-0.6B: 28 layers, hidden 1024, FFN 3072, 16 q / 8 kv heads x 128, vocab 151936, tied head."""
    attn = ModelConfig(28, 16, 8, 128, RotaryConfig(128, 128, 1e6, 40960), hidden_size=1024)
    return Qwen3Spec(attn, 1024, 3072, 151936)


def tiny_spec(num_layers: int = 2, vocab_size: int = 512) -> Qwen3Spec:
    """A small model of the same structure for parity tests (16 q / 8 kv heads x 128)."""
    attn = ModelConfig(num_layers, 16, 8, 128, RotaryConfig(128, 128, 1e6, 40960), hidden_size=256)
    return Qwen3Spec(attn, 256, 512, vocab_size)


class _Layer:
    def __init__(self, spec: Qwen3Spec, layer_id: int, gen: torch.Generator, dtype, device) -> None:
        a = spec.attn
        H, D = spec.hidden_size, a.head_dim
        qkv = (a.num_qo_heads + 2 * a.num_kv_heads) * D

        def w(o, i):
            return (torch.randn((o, i), generator=gen, device=device, dtype=torch.float32) * 0.02).to(dtype)

        self.in_norm = torch.ones(H, dtype=dtype, device=device)
        self.qkv = w(qkv, H)
        self.q_norm = torch.ones(D, dtype=dtype, device=device)
        self.k_norm = torch.ones(D, dtype=dtype, device=device)
        self.o = w(H, a.num_qo_heads * D)
        self.post_norm = torch.ones(H, dtype=dtype, device=device)
        self.gate_up = w(2 * spec.intermediate_size, H)
        self.down = w(H, spec.intermediate_size)
        self.attn = AttentionLayer(layer_id, a.num_qo_heads, a.num_kv_heads, D, a.rotary_config)


class Qwen3Model:
    def __init__(self, spec: Qwen3Spec, dtype: torch.dtype, device: torch.device, seed: int = 42) -> None:
        self.spec = spec
        gen = torch.Generator(device=device).manual_seed(seed)
        self.embed = (torch.randn((spec.vocab_size, spec.hidden_size), generator=gen, device=device,
                                  dtype=torch.float32) * 0.02).to(dtype)
        with torch.cuda.device(device):
            self.layers: List[_Layer] = [_Layer(spec, i, gen, dtype, device) for i in range(spec.attn.num_layers)]
        self.norm = torch.ones(spec.hidden_size, dtype=dtype, device=device)
        # b2a_proj shapes: bf16, K (hidden, heads x head_dim, intermediate) multiples of 128
        a = spec.attn
        self.fused_proj = (dtype == torch.bfloat16 and spec.hidden_size % 128 == 0
                           and (a.num_qo_heads * a.head_dim) % 128 == 0 and spec.intermediate_size % 128 == 0)

    @property
    def nbytes(self) -> int:
        ts = [self.embed, self.norm]
        for L in self.layers:
            ts += [L.in_norm, L.qkv, L.q_norm, L.k_norm, L.o, L.post_norm, L.gate_up, L.down]
        return sum(t.numel() * t.element_size() for t in ts)

    def __call__(self, input_ids: torch.Tensor) -> torch.Tensor:
        """input_ids ``[T]`` -> logits ``[B, vocab]`` of each request's last token."""
        spec, a = self.spec, self.spec.attn
        Hq, Hkv, D, eps = a.num_qo_heads, a.num_kv_heads, a.head_dim, spec.rms_norm_eps
        batch = get_global_ctx().batch
        h = F.embedding(input_ids, self.embed)
        T = h.shape[0]
        if self.fused_proj and T <= FUSED_MAX_ROWS:
            for L in self.layers:
                qkv = proj(h, L.qkv, PROJ_PLAIN, L.in_norm, eps)
                q = qkv[:, : Hq * D].view(T, Hq, D)
                k = qkv[:, Hq * D: (Hq + Hkv) * D].view(T, Hkv, D)
                v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
                proj(L.attn(q, k, v, L.q_norm, L.k_norm, eps), L.o, PROJ_RESIDUAL, res=h, out=h)
                proj(proj(h, L.gate_up, PROJ_SWIGLU, L.post_norm, eps), L.down, PROJ_RESIDUAL, res=h, out=h)
            h = rms_norm(h, self.norm, eps, batch.attn_metadata.last_indices if batch.is_prefill else None)
            return F.linear(h, self.embed)
        for L in self.layers:
            x = rms_norm(h, L.in_norm, eps)
            qkv = F.linear(x, L.qkv)
            q = qkv[:, : Hq * D].view(T, Hq, D)
            k = qkv[:, Hq * D: (Hq + Hkv) * D].view(T, Hkv, D)
            v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
            # q/k RMSNorm fused into the RoPE + KV-store kernel
            h = torch.addmm(h, L.attn(q, k, v, L.q_norm, L.k_norm, eps), L.o.t())
            x = rms_norm(h, L.post_norm, eps)
            h = torch.addmm(h, swiglu(F.linear(x, L.gate_up)), L.down.t())
        # prefill: only each request's last token is normed and projected (one gather + norm kernel)
        h = rms_norm(h, self.norm, eps, batch.attn_metadata.last_indices if batch.is_prefill else None)
        return F.linear(h, self.embed)
