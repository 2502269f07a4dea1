"""Shared test setup.

* registers the ``gpu`` marker: GPU tests run on a B200 via ``pytest -m gpu``;
  everything else runs on the CPU (``-m "not gpu"``).
* puts the package directory (mini-sglang-mlx_b200/) and the repo root (for
  oracle/) on sys.path.
* a GPU test on a host without CUDA FAILS (it never silently skips), so a GPU
  run cannot pass on a fallback.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "mini-sglang-mlx_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_runtest_setup(item):
    if item.get_closest_marker("gpu") is not None:
        import torch

        if not torch.cuda.is_available():
            pytest.fail("GPU test collected on a host without CUDA (run with -m 'not gpu' on CPU)")


@pytest.fixture(autouse=True)
def reset_global_ctx():
    import minisgl_b200.core as core

    old = core._GLOBAL_CTX
    yield
    core._GLOBAL_CTX = old
