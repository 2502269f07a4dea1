"""Integer helpers with the reference's semantics (python/minisgl_mlx/utils.py:37-46)."""

from __future__ import annotations


def div_ceil(a: int, b: int) -> int:
    return (a + b - 1) // b


def align_down(a: int, b: int) -> int:
    return a // b * b


def align_up(a: int, b: int) -> int:
    return div_ceil(a, b) * b
