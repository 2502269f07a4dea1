"""CPU oracle of the engine harness's generation -- TEST INFRASTRUCTURE ONLY.

Greedy generation by full recomputation: for every request, every step runs
the whole sequence through the model in float64 and appends the argmax of the
last position. No KV cache, no batching, no paging, no scheduler -- so
tokens identical to the engine harness pin its scheduling, chunked prefill,
prefix reuse, paging and the attention path together.

The forward restates python/minisgl_mlx/models/transformer.py:33-116 (RMSNorm,
fused qkv, per-head q/k RMSNorm, rotate-half RoPE from layers.py:45-56 via
``attention.rope``, causal softmax attention with GQA, o_proj, SwiGLU MLP,
final RMSNorm, tied embedding head) and engine/sample.py:51-55 (greedy =
argmax). Weights are read from a ``minisgl_b200.engine.Qwen3Model``.
"""

from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np

from . import attention as O


def _np(t) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def _rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


class OracleQwen3:
    def __init__(self, model) -> None:
        spec = model.spec
        a = spec.attn
        self.Hq, self.Hkv, self.D = a.num_qo_heads, a.num_kv_heads, a.head_dim
        self.eps = spec.rms_norm_eps
        self.dims = a.rotary_config.rotary_dim
        self.inv_freq = O.rope_inv_freq(self.dims, a.rotary_config.base).astype(np.float64)
        self.embed = _np(model.embed)
        self.norm = _np(model.norm)
        self.layers: List[Dict[str, np.ndarray]] = []
        for L in model.layers:
            self.layers.append({k: _np(getattr(L, k)) for k in
                                ("in_norm", "qkv", "q_norm", "k_norm", "o", "post_norm", "gate_up", "down")})

    def logits_last(self, ids: Sequence[int]) -> np.ndarray:
        """Logits of the last position of the sequence ``ids``."""
        Hq, Hkv, D = self.Hq, self.Hkv, self.D
        G = Hq // Hkv
        T = len(ids)
        pos = np.arange(T)
        h = self.embed[np.asarray(ids)]
        causal = np.tril(np.ones((T, T), dtype=bool))
        for W in self.layers:
            x = _rms(h, W["in_norm"], self.eps)
            qkv = x @ W["qkv"].T
            q = _rms(qkv[:, : Hq * D].reshape(T, Hq, D), W["q_norm"], self.eps)
            k = _rms(qkv[:, Hq * D: (Hq + Hkv) * D].reshape(T, Hkv, D), W["k_norm"], self.eps)
            v = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
            q = O.rope(q, pos, self.dims, self.inv_freq)
            k = O.rope(k, pos, self.dims, self.inv_freq)
            o = np.empty((T, Hq, D))
            for hq in range(Hq):
                s = (q[:, hq, :] @ k[:, hq // G, :].T) * D ** -0.5
                s = np.where(causal, s, -np.inf)
                p = np.exp(s - s.max(axis=1, keepdims=True))
                p /= p.sum(axis=1, keepdims=True)
                o[:, hq, :] = p @ v[:, hq // G, :]
            h = h + o.reshape(T, Hq * D) @ W["o"].T
            x = _rms(h, W["post_norm"], self.eps)
            gu = x @ W["gate_up"].T
            gate, up = np.split(gu, 2, axis=-1)
            h = h + (gate / (1.0 + np.exp(-gate)) * up) @ W["down"].T
        hl = _rms(h[-1:], self.norm, self.eps)
        return (hl @ self.embed.T)[0]

    def generate(self, prompts: Sequence[Sequence[int]], max_tokens: Sequence[int]) -> List[List[int]]:
        out = []
        for p, n in zip(prompts, max_tokens):
            seq = list(int(t) for t in p)
            gen = []
            for _ in range(n):
                tok = int(np.argmax(self.logits_last(seq)))
                gen.append(tok)
                seq.append(tok)
            out.append(gen)
        return out
