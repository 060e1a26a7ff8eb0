"""CPU oracle for the vector pipeline.  TEST INFRASTRUCTURE ONLY.

Restates ``examples/vector_pipeline.py:17-24``: two chained launches of
``update`` (``dst[i] = src[i] + bias``, ``:9-14``) through an ``empty_like`` temporary, so
``dst = (src + bias) + bias`` with two float32 roundings.  The fused form computes the same
two rounded additions (no reassociation into ``src + 2*bias``).
"""
from __future__ import annotations

import numpy as np


def make_source(n: int, seed: int = 1) -> np.ndarray:
    """``src ~ U(-1, 1)`` float32 from ``default_rng(seed)``."""
    return np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32)


def pipeline(src: np.ndarray, bias: float, out: np.ndarray | None = None) -> np.ndarray:
    b = np.float32(bias)
    if out is None:
        out = np.empty_like(src)
    np.add(src, b, out=out)
    np.add(out, b, out=out)
    return out
