"""End-to-end engine harness: random-init Qwen3 over the B200 attention backend.

Re-hosts the call surface of the reference's engine, scheduler and offline
LLM (python/minisgl_mlx/{engine,scheduler,kvcache/radix_cache,llm}.py) so that
the attention path runs inside a serving loop: chunked prefill with a radix
prefix cache, continuous decode and overlap scheduling.
"""

from .managers import CacheManager, ChunkedReq, DecodeManager, PendingReq, PrefillManager, TableManager
from .model import Qwen3Model, Qwen3Spec, qwen3_0_6b_spec, tiny_spec
from .radix import NaivePrefixCache, PrefixHandle, RadixPrefixCache, create_prefix_cache
from .router import prefix_key, route_requests
from .scheduler import LLM, Engine, EngineConfig, HostScheduler, Scheduler

__all__ = [
    "CacheManager", "ChunkedReq", "DecodeManager", "Engine", "EngineConfig", "LLM", "NaivePrefixCache",
    "HostScheduler", "PendingReq", "PrefillManager", "PrefixHandle", "Qwen3Model", "Qwen3Spec", "RadixPrefixCache",
    "Scheduler", "TableManager", "create_prefix_cache", "prefix_key", "qwen3_0_6b_spec", "route_requests",
    "tiny_spec",
]
