"""RoPE set-up pinned to the reference's own code (CPU).

tests/golden/rope_tables_ref.npz was made by running the reference's
RotaryEmbedding.__init__ and _llama3_freqs (python/minisgl_mlx/layers.py:28-74)
with a numpy stand-in for the mlx.core calls they make (generator:
tests/golden/make_golden_rope.py). Our host tables must give the same rope
arguments: the position scale (1 / factor for linear scaling), the base, and
the llama3 period table bit for bit. The rotation itself (mx.fast.rope) is MLX
library code that cannot run here; it is covered by the known-answer tests.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

import make_golden_rope as GR  # noqa: E402

FIXTURE = Path(__file__).resolve().parent / "golden" / "rope_tables_ref.npz"


@pytest.fixture(scope="module")
def golden():
    return np.load(FIXTURE)


@pytest.mark.parametrize("name", [c[0] for c in GR.CASES])
def test_rope_tables_match_reference_setup(golden, name):
    from minisgl_b200.config import RotaryConfig
    from minisgl_b200.layers import llama3_freqs, rope_tables

    fields = json.loads(str(golden[f"{name}_config"]))
    assert fields == dict(GR.CASES)[name]
    inv, scale = rope_tables(RotaryConfig(**fields))
    assert scale == float(golden[f"{name}_scale"])
    assert inv.shape == (int(golden[f"{name}_dims"]) // 2,)
    ref_freqs = golden[f"{name}_freqs"]
    if ref_freqs.size:  # llama3: the reference passes freqs=..., base=None
        assert np.isnan(float(golden[f"{name}_base"]))
        ours = llama3_freqs(fields["rotary_dim"], fields["base"], fields["scaling"])
        assert ours.dtype == np.float32
        np.testing.assert_array_equal(ours, ref_freqs)
        np.testing.assert_array_equal(inv, np.float32(1.0) / ref_freqs)
    else:
        assert float(golden[f"{name}_base"]) == fields["base"]


def test_reference_setup_reproduces_fixture(golden):
    ref = os.environ.get("MINISGL_REFERENCE") or str(Path(__file__).resolve().parents[2] / "reference")
    ref = Path(ref)
    if not (ref / "python" / "minisgl_mlx" / "layers.py").exists():
        pytest.skip("no reference checkout on this host")
    layers, config = GR.load_reference_layers(ref)
    for name, fields in GR.CASES:
        rope = layers.RotaryEmbedding(config.RotaryConfig(**fields))
        assert float(rope.scale) == float(golden[f"{name}_scale"])
        if rope.freqs is not None:
            np.testing.assert_array_equal(np.asarray(rope.freqs), golden[f"{name}_freqs"])
