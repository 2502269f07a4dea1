"""Generate tests/golden/rope_tables_ref.npz from the reference's own RoPE set-up code.

The reference's RotaryEmbedding (python/minisgl_mlx/layers.py:28-56) turns a
RotaryConfig into the arguments of mx.fast.rope: `dims`, `base`, the position
`scale` (1 / factor for linear scaling, layers.py:37-38) and, for llama3
scaling, a table of rotary periods computed by `_llama3_freqs`
(layers.py:59-74). That set-up is plain array arithmetic, so this script runs
the reference's own layers.py -- loaded from a reference checkout, never
copied -- with a small numpy stand-in for the few `mlx.core` calls it makes
(`arange`, `where`; array operators keep MLX's float32 promotion: an int32
range divided by an int is float32, a Python scalar never widens a float32
array). The rotation itself, inside mx.fast.rope, is MLX library code and is
not run here.

Stored per case: dims, base (NaN when the reference passes base=None), scale,
and the period table (float32, empty when there is none).

    python tests/golden/make_golden_rope.py --reference <mini-sglang-mlx checkout>
    (or MINISGL_REFERENCE=<checkout> python tests/golden/make_golden_rope.py)
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "rope_tables_ref.npz"

# (name, RotaryConfig fields): Qwen3 default, linear scaling, Llama 3.1 and Llama 3.2 style llama3 scaling
CASES = [
    ("qwen3_default", dict(head_dim=128, rotary_dim=128, base=1000000.0, max_position=40960, scaling=None)),
    ("linear_x4", dict(head_dim=128, rotary_dim=128, base=10000.0, max_position=16384,
                       scaling={"rope_type": "linear", "factor": 4.0})),
    ("llama31", dict(head_dim=128, rotary_dim=128, base=500000.0, max_position=131072,
                     scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                              "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})),
    ("llama32_d64", dict(head_dim=64, rotary_dim=64, base=500000.0, max_position=131072,
                         scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                  "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})),
]


class _IntRange(np.ndarray):
    """An int32 array whose true division gives float32, as an MLX int32 array's does."""

    def __truediv__(self, other):
        return np.true_divide(self.view(np.ndarray), other, dtype=np.float32)


def _mlx_core_stub() -> types.ModuleType:
    core = types.ModuleType("mlx.core")

    def arange(start, stop=None, step=1):
        if stop is None:
            start, stop = 0, start
        return np.arange(start, stop, step, dtype=np.int32).view(_IntRange)

    def where(cond, a, b):
        return np.where(cond, a, b)

    core.arange = arange
    core.where = where
    core.array = lambda x, dtype=None: np.asarray(x, dtype=np.float32)
    return core


def load_reference_layers(reference: Path):
    """Import the reference's layers.py (and models/config.py) with stand-ins for mlx."""
    pkg = reference / "python" / "minisgl_mlx"
    mlx = types.ModuleType("mlx")
    mlx.__path__ = []
    core = _mlx_core_stub()
    mlx.core = core
    ctx = types.ModuleType("minisgl_mlx.core")
    ctx.get_global_ctx = lambda: None  # only AttentionLayer uses it; not called here
    saved = {k: sys.modules.get(k) for k in ("mlx", "mlx.core", "minisgl_mlx", "minisgl_mlx.core",
                                               "minisgl_mlx.models", "minisgl_mlx.models.config")}
    try:
        sys.modules["mlx"], sys.modules["mlx.core"] = mlx, core
        root = types.ModuleType("minisgl_mlx")
        root.__path__ = [str(pkg)]
        models = types.ModuleType("minisgl_mlx.models")
        models.__path__ = [str(pkg / "models")]
        sys.modules["minisgl_mlx"], sys.modules["minisgl_mlx.models"] = root, models
        sys.modules["minisgl_mlx.core"] = ctx
        cspec = importlib.util.spec_from_file_location("minisgl_mlx.models.config", pkg / "models" / "config.py")
        cmod = importlib.util.module_from_spec(cspec)
        sys.modules["minisgl_mlx.models.config"] = cmod
        cspec.loader.exec_module(cmod)
        lspec = importlib.util.spec_from_file_location("_reference_layers", pkg / "layers.py")
        lmod = importlib.util.module_from_spec(lspec)
        lspec.loader.exec_module(lmod)
        return lmod, cmod
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    args = ap.parse_args()
    ref = args.reference or (Path(os.environ["MINISGL_REFERENCE"]) if os.environ.get("MINISGL_REFERENCE") else None)
    if ref is None or not (ref / "python" / "minisgl_mlx" / "layers.py").exists():
        raise SystemExit("name the reference checkout with --reference or MINISGL_REFERENCE")
    layers, config = load_reference_layers(ref)
    data = {}
    for name, fields in CASES:
        rope = layers.RotaryEmbedding(config.RotaryConfig(**fields))
        data[f"{name}_config"] = np.array(json.dumps(fields))
        data[f"{name}_dims"] = np.array(rope.dims)
        data[f"{name}_base"] = np.array(np.nan if rope.base is None else float(rope.base))
        data[f"{name}_scale"] = np.array(float(rope.scale))
        freqs = np.zeros(0, np.float32) if rope.freqs is None else np.asarray(rope.freqs)
        assert freqs.dtype == np.float32
        data[f"{name}_freqs"] = freqs
    np.savez_compressed(OUT, **data)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
