"""minisgl_b200 - a B200-native attention backend for mini-sglang-mlx.

Importing the package loads the CUDA library (libb200attn.so) and fails
loudly if it is missing; there is no fallback implementation.
"""

from . import _native
from .attention import (
    SUPPORTED_ATTENTION_BACKENDS,
    B200AttnBackend,
    BaseAttnBackend,
    create_attention_backend,
    paged_decode_attention,
)
from .config import ModelConfig, RotaryConfig
from .core import Batch, Context, Req, get_global_ctx, set_global_ctx
from .kvcache import MHAKVCache
from .layers import AttentionLayer, RotaryEmbedding

__all__ = [
    "AttentionLayer",
    "B200AttnBackend",
    "BaseAttnBackend",
    "Batch",
    "Context",
    "MHAKVCache",
    "ModelConfig",
    "Req",
    "RotaryConfig",
    "RotaryEmbedding",
    "SUPPORTED_ATTENTION_BACKENDS",
    "create_attention_backend",
    "get_global_ctx",
    "paged_decode_attention",
    "set_global_ctx",
]
