"""Backend registry with the reference's selection contract.

Mirrors python/minisgl_mlx/attention/__init__.py:15-26: ``--attn`` choices are
the keys of SUPPORTED_ATTENTION_BACKENDS and an unknown name raises
ValueError with the same message shape.
"""

from __future__ import annotations

from .b200 import B200AttnBackend, B200DecodeMetadata, B200PrefillMetadata, page_table_scatter, paged_decode_attention
from .base import BaseAttnBackend, PinnedStager, paged_kv_indices

SUPPORTED_ATTENTION_BACKENDS = {
    "b200": B200AttnBackend,  # CUDA sm_100a kernels: split-KV paged decode, tcgen05 extend
}


def create_attention_backend(name: str, config, kv_cache, page_table) -> BaseAttnBackend:
    if name not in SUPPORTED_ATTENTION_BACKENDS:
        raise ValueError(f"Unknown attention backend {name!r}: {list(SUPPORTED_ATTENTION_BACKENDS)}")
    return SUPPORTED_ATTENTION_BACKENDS[name](config, kv_cache, page_table)


__all__ = [
    "BaseAttnBackend",
    "B200AttnBackend",
    "B200DecodeMetadata",
    "B200PrefillMetadata",
    "PinnedStager",
    "SUPPORTED_ATTENTION_BACKENDS",
    "create_attention_backend",
    "paged_decode_attention",
    "page_table_scatter",
    "paged_kv_indices",
]
