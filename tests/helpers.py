"""Shared helpers for the GPU parity tests."""

from __future__ import annotations

import numpy as np

from oracle import attention as O

# BASELINE tolerances: max-abs against an fp64/fp32 reference
TOL = {"float32": 1e-5, "bfloat16": 2e-2}


def torch_dtype(name: str):
    import torch

    return {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[name]


def rand(rng: np.random.Generator, shape, dtype: str) -> np.ndarray:
    """N(0,1) values already rounded to `dtype` (float32 carrier)."""
    return O.round_to(rng.standard_normal(shape).astype(np.float32), dtype)


def to_dev(a: np.ndarray, dtype: str):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=torch_dtype(dtype))


def to_np(t) -> np.ndarray:
    import torch

    return t.detach().to(torch.float32).cpu().numpy().astype(np.float64)


def max_abs(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if a.size else 0.0


class HeadConfig:
    def __init__(self, Hq: int, Hkv: int, D: int):
        self.num_qo_heads = Hq
        self.num_kv_heads = Hkv
        self.head_dim = D
