"""ctypes wrapper of oracle/_ref/libmetal_ref.so -- TEST INFRASTRUCTURE ONLY.

``metal_paged_decode`` runs the reference's own Metal paged-decode kernel body
(python/minisgl_mlx/attention/metal.py:35-95) on the CPU with the launch
geometry of paged_decode_attention (metal.py:112-131). bf16 tensors travel as
float32 arrays holding bf16 values and are converted to bf16 bit patterns here.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parents[1] / "_ref" / "libmetal_ref.so"
_lib = None


def available() -> bool:
    return LIB_PATH.exists()


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        I = ctypes.c_int
        _lib.metal_ref_paged_decode.argtypes = [P, P, P, P, P, ctypes.c_float, I, I, I, I, I, I, P]
        _lib.metal_ref_paged_decode.restype = I
    return _lib


def _as_dtype(a: np.ndarray, dtype: str) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    if dtype == "float32":
        return a
    # float32 carrier holding bf16 values -> the bf16 bit pattern (exact)
    return np.ascontiguousarray((a.view(np.uint32) >> 16).astype(np.uint16))


def metal_paged_decode(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, kv_indptr: np.ndarray,
                       kv_indices: np.ndarray, scale: float, dtype: str) -> np.ndarray:
    """q [B,Hq,D], pools [N,Hkv,D] -> out [B,Hq,D] as float32 (bf16 values when dtype is bfloat16)."""
    lib = _load()
    B, Hq, D = q.shape
    N, Hkv, _ = k_pool.shape
    code = 0 if dtype == "float32" else 1
    qq, kk, vv = _as_dtype(q, dtype), _as_dtype(k_pool, dtype), _as_dtype(v_pool, dtype)
    out = np.zeros(q.shape, dtype=np.float32 if code == 0 else np.uint16)
    ind = np.ascontiguousarray(kv_indptr, dtype=np.int32)
    idx = np.ascontiguousarray(kv_indices, dtype=np.int32)
    rc = lib.metal_ref_paged_decode(qq.ctypes.data, kk.ctypes.data, vv.ctypes.data, ind.ctypes.data,
                                    idx.ctypes.data, float(scale), B, Hq, Hkv, N, D, code, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"metal_ref_paged_decode returned {rc}")
    if code == 0:
        return out
    return (out.astype(np.uint32) << 16).view(np.float32)
