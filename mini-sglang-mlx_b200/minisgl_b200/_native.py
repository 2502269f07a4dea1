"""ctypes binding of the C ABI in include/b200attn.h (libb200attn.so).

This module is the only place that talks to the shared library. Device
pointers go in as integers (``tensor.data_ptr()``), streams as the raw
``cudaStream_t`` value of torch's current stream. Every call checks the
returned status and raises with the library's own message; there is no
fallback path: if the library cannot be loaded, importing this module fails.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import numpy as np

LIB_NAME = "libb200attn.so"
LIB_PATH = Path(os.environ.get("MINISGL_B200_LIB", Path(__file__).resolve().parent / LIB_NAME))

B2A_DTYPE_F32 = 0
B2A_DTYPE_BF16 = 1
B2A_DTYPE_F16 = 2

B2A_OK = 0
B2A_ERR_INVALID = 1
B2A_ERR_UNSUPPORTED = 2
B2A_ERR_CUDA = 3
B2A_ERR_WORKSPACE = 4

_P = c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)

# name -> (restype, argtypes); mirrors include/b200attn.h one to one.
SIGNATURES = {
    "b2a_last_error": (ctypes.c_char_p, []),
    "b2a_abi_version": (c_int, []),
    "b2a_device_error": (c_int, [_P, ctypes.POINTER(c_int)]),
    "b2a_store_kv": (
        c_int,
        [_P, c_int64, _P, c_int64, _P, _P, _P, c_int64, c_int, c_int, c_int, c_int, _P],
    ),
    "b2a_rope_store": (
        c_int,
        [_P, c_int64, _P, c_int64, _P, c_int64, _P, _P, _P, _P, c_int64, _P, c_float, c_int,
         c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "b2a_qknorm_rope_store": (
        c_int,
        [_P, c_int64, _P, _P, c_int64, _P, c_int64, _P, _P, c_float, _P, _P, _P, _P, c_int64, _P, c_float, c_int,
         c_int, c_int, c_int, c_int, c_int, _P],
    ),
    "b2a_paged_decode": (
        c_int,
        [_P, _P, _P, c_int64, _P, _P, c_int, c_int, c_int, c_int, c_float, _P, c_int, _P],
    ),
    "b2a_decode_plan": (
        c_int,
        [_P, _P, c_int, c_int, c_int, _P, _P, c_int, _P, ctypes.POINTER(c_int),
         ctypes.POINTER(c_int)],
    ),
    "b2a_decode_metadata": (
        c_int,
        [_P, c_int64, c_int64, _P, _P, c_int, c_int, c_int, _P, _P, c_int64, _P, _P, _P, c_int, _P, _P, _P],
    ),
    "b2a_page_table_scatter": (c_int, [_P, c_int64, c_int64, _P, _P, _P, c_int64, _P]),
    "b2a_decode_num_ctas": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(c_int)]),
    "b2a_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "b2a_decode": (
        c_int,
        [_P, _P, _P, c_int64, _P, c_int, _P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_float,
         _P, c_size_t, _P, c_int, _P],
    ),
    "b2a_decode_noalloc": (
        c_int,
        [_P, _P, _P, c_int64, _P, c_int, _P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_float,
         _P, c_int, _P],
    ),
    "b2a_extend_tile_q": (c_int, [c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(c_int)]),
    "b2a_pack_kv": (
        c_int,
        [_P, _P, c_int64, _P, _P, c_int, _P, _P, c_int, c_int64, c_int, c_int, c_int, _P, _P, c_int64, _P],
    ),
    "b2a_extend_plan": (
        c_int,
        [_P, _P, _P, c_int, c_int, c_int, _P, c_int, ctypes.POINTER(c_int)],
    ),
    "b2a_extend": (
        c_int,
        [_P, _P, _P, c_int64, _P, _P, _P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, _P, c_int, _P],
    ),
    "b2a_extend_groups": (
        c_int,
        [_P, _P, _P, c_int64, _P, _P, c_int64, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int,
         c_float, _P, c_int, _P],
    ),
    "b2a_swiglu": (c_int, [_P, c_int64, _P, c_int64, c_int, c_int, _P]),
    "b2a_rmsnorm": (c_int, [_P, c_int64, c_int64, _P, c_int64, _P, c_float, c_int, _P, c_int, _P]),
    "b2a_proj": (c_int, [_P, c_int64, c_int, c_int, _P, c_int, _P, c_float, _P, c_int64, _P, c_int64, c_int, c_int,
                         _P]),
}


class B200AttnError(RuntimeError):
    """A C-ABI call returned a nonzero status."""

    def __init__(self, fn: str, code: int, msg: str) -> None:
        super().__init__(f"{fn} failed (code {code}): {msg}")
        self.code = code


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python mini-sglang-mlx_b200/build.py` "
            "(the B200 attention backend has no non-CUDA fallback)"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def last_error() -> str:
    return (LIB.b2a_last_error() or b"").decode()


def call(name: str, *args) -> None:
    """Call an int-status entry point and raise B200AttnError on failure."""
    rc = getattr(LIB, name)(*args)
    if rc != B2A_OK:
        err = last_error()
        if rc == B2A_ERR_INVALID:
            raise ValueError(f"{name}: {err}")
        raise B200AttnError(name, rc, err)


def np_ptr(a: np.ndarray | None) -> int | None:
    """Host pointer of a C-contiguous int32 numpy array (None passes NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"] and a.dtype == np.int32, (a.dtype, a.flags)
    return a.ctypes.data


def decode_plan(kv_indptr: np.ndarray, kv_last_page_len: np.ndarray | None, page_size: int,
                num_ctas: int):
    """Host-side split plan (b2a_decode_plan). Returns (cta_indptr, segs, merge_indptr, n_partials)."""
    kv_indptr = np.ascontiguousarray(kv_indptr, dtype=np.int32)
    B = kv_indptr.shape[0] - 1
    lpl = None if kv_last_page_len is None else np.ascontiguousarray(kv_last_page_len, dtype=np.int32)
    cap = B + num_ctas + 1
    cta_indptr = np.zeros(num_ctas + 1, np.int32)
    segs = np.zeros(cap * 4, np.int32)
    merge_indptr = np.zeros(B + 1, np.int32)
    n_segs, n_part = c_int(0), c_int(0)
    call("b2a_decode_plan", np_ptr(kv_indptr), np_ptr(lpl), B, page_size, num_ctas,
         np_ptr(cta_indptr), np_ptr(segs), cap, np_ptr(merge_indptr), ctypes.byref(n_segs),
         ctypes.byref(n_part))
    return cta_indptr, segs[: 4 * n_segs.value].reshape(-1, 4), merge_indptr, n_part.value


def extend_tile_q(Hq: int, Hkv: int, D: int, dtype_code: int, page_size: int) -> int:
    t = c_int(0)
    call("b2a_extend_tile_q", Hq, Hkv, D, dtype_code, page_size, ctypes.byref(t))
    return t.value


def extend_plan(qo_indptr: np.ndarray, kv_indptr: np.ndarray, kv_last_page_len: np.ndarray | None,
                page_size: int, tile_q: int) -> np.ndarray:
    """Host-side tile list (b2a_extend_plan): int32 [n_work, 4], longest tiles first."""
    qo = np.ascontiguousarray(qo_indptr, dtype=np.int32)
    kv = np.ascontiguousarray(kv_indptr, dtype=np.int32)
    lpl = None if kv_last_page_len is None else np.ascontiguousarray(kv_last_page_len, dtype=np.int32)
    B = qo.shape[0] - 1
    total_q = int(qo[-1]) if B > 0 else 0
    cap = max(1, B + total_q // max(tile_q, 1) + 1)
    work = np.zeros(cap * 4, np.int32)
    n = c_int(0)
    call("b2a_extend_plan", np_ptr(qo), np_ptr(kv), np_ptr(lpl), B, page_size, tile_q,
         np_ptr(work), cap, ctypes.byref(n))
    return work[: 4 * n.value].reshape(-1, 4)


def decode_workspace_bytes(n_partials: int, Hq: int, D: int) -> int:
    return int(LIB.b2a_decode_workspace_bytes(n_partials, Hq, D))
