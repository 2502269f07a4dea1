"""Model-shape configuration read by the attention path.

Field names follow python/minisgl_mlx/models/config.py:9-35 (RotaryConfig,
ModelConfig). Only what the attention backend, the pool and the rotary
embedding need is kept; `from_hf` parses the same HF config keys as
models/config.py:37-78.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict


@dataclass(frozen=True)
class RotaryConfig:
    head_dim: int
    rotary_dim: int
    base: float
    max_position: int
    scaling: Dict[str, Any] | None = None


@dataclass(frozen=True)
class ModelConfig:
    num_layers: int
    num_qo_heads: int
    num_kv_heads: int
    head_dim: int
    rotary_config: RotaryConfig
    hidden_size: int = 0
    model_type: str = "qwen3"

    @classmethod
    def from_hf(cls, cfg: Dict[str, Any]) -> "ModelConfig":
        num_qo_heads = cfg["num_attention_heads"]
        hidden = cfg["hidden_size"]
        head_dim = cfg.get("head_dim") or hidden // num_qo_heads
        rope_params = cfg.get("rope_parameters") or {}
        theta = cfg.get("rope_theta", rope_params.get("rope_theta", 10000.0))
        scaling = cfg.get("rope_scaling") or None
        if scaling is None and rope_params.get("rope_type", "default") != "default":
            scaling = rope_params
        return cls(
            num_layers=cfg["num_hidden_layers"],
            num_qo_heads=num_qo_heads,
            num_kv_heads=cfg.get("num_key_value_heads", num_qo_heads),
            head_dim=head_dim,
            hidden_size=hidden,
            model_type=cfg.get("model_type", "llama"),
            rotary_config=RotaryConfig(
                head_dim=head_dim,
                rotary_dim=int(head_dim * cfg.get("partial_rotary_factor", 1.0)),
                base=float(theta),
                max_position=cfg.get("max_position_embeddings", 4096),
                scaling=scaling,
            ),
        )


def qwen3_0_6b() -> ModelConfig:
    """Attention shape of Qwen3-0.6B (28 layers, 16 q / 8 kv heads, head_dim 128, theta 1e6)."""
    return ModelConfig(28, 16, 8, 128, RotaryConfig(128, 128, 1e6, 40960), hidden_size=1024)


def qwen3_8b() -> ModelConfig:
    """Attention shape of Qwen3-8B (36 layers, 32 q / 8 kv heads, head_dim 128, theta 1e6)."""
    return ModelConfig(36, 32, 8, 128, RotaryConfig(128, 128, 1e6, 40960), hidden_size=4096)
