"""KV pool on the GPU with the reference's interface.

Mirrors MHAKVCache (python/minisgl_mlx/kvcache/pool.py:24-54):
``k[layer]`` / ``v[layer]`` are ``[num_tokens, num_kv_heads, head_dim]``, zero
initialised, and a slot is the first index. HBM layout: ONE allocation
``[num_layers, 2, num_tokens, Hkv, D]`` so that a slot row (all kv heads of
one token, 2 KB for 8 x 128 bf16) and a page (page_size consecutive rows) are
contiguous for bulk copies, and K and V of a layer are adjacent. ``k``/``v``
are per-layer views of it.

``store_kv`` is the CUDA scatter kernel (b2a_store_kv), byte-exact.
"""

from __future__ import annotations

from typing import List

import torch

from .. import _native as nat

_DTYPE_CODE = {
    torch.float32: nat.B2A_DTYPE_F32,
    torch.bfloat16: nat.B2A_DTYPE_BF16,
    torch.float16: nat.B2A_DTYPE_F16,
}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError as e:
        raise ValueError(f"unsupported dtype {dtype}") from e


def current_stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class MHAKVCache:
    def __init__(
        self,
        num_layers: int,
        num_tokens: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device | str | None = None,
    ) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("MHAKVCache needs a CUDA device (no CPU fallback)")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.buffer = torch.zeros(
            (num_layers, 2, num_tokens, num_kv_heads, head_dim), dtype=dtype, device=device
        )
        self.k: List[torch.Tensor] = [self.buffer[l, 0] for l in range(num_layers)]
        self.v: List[torch.Tensor] = [self.buffer[l, 1] for l in range(num_layers)]
        self.num_layers = num_layers
        self.num_tokens = num_tokens
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device

    def k_cache(self, layer_id: int) -> torch.Tensor:
        return self.k[layer_id]

    def v_cache(self, layer_id: int) -> torch.Tensor:
        return self.v[layer_id]

    def store_kv(self, k: torch.Tensor, v: torch.Tensor, out_loc: torch.Tensor, layer_id: int) -> None:
        """Write k/v ``[T, Hkv, D]`` into slots ``out_loc`` ``[T]`` (kvcache/pool.py:47-50)."""
        T = k.shape[0]
        assert k.shape == v.shape == (T, self.num_kv_heads, self.head_dim), (k.shape, v.shape)
        assert k.dtype == v.dtype == self.dtype
        assert out_loc.dtype == torch.int32 and out_loc.is_cuda and out_loc.numel() == T
        assert k.stride(2) == 1 and k.stride(1) == self.head_dim, "k rows must be [Hkv, D] contiguous"
        assert v.stride(2) == 1 and v.stride(1) == self.head_dim, "v rows must be [Hkv, D] contiguous"
        nat.call(
            "b2a_store_kv", k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
            out_loc.data_ptr(), self.k[layer_id].data_ptr(), self.v[layer_id].data_ptr(),
            self.num_tokens, T, self.num_kv_heads, self.head_dim, dtype_code(self.dtype),
            current_stream_ptr(self.device),
        )

    @property
    def nbytes(self) -> int:
        return self.buffer.numel() * self.buffer.element_size()
