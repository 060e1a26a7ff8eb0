"""Request sharding across GPUs: contiguous request ranges, one process per GPU.

Decode requests never interact (every buffer but the read-only weights is per request), so a
job of R requests on G GPUs gives rank r the contiguous range ``request_range(R, G, r)`` with a
full weight replica and its own KV cache, tokens and history; no collective runs in the step.
Prompts are drawn for the whole job and sliced, so a request's prompt does not depend on G.
"""
from __future__ import annotations

import numpy as np


def request_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's requests: ceil(total / world) per rank, the last may be short."""
    if world <= 0 or not 0 <= rank < world or total <= 0:
        raise ValueError("need total > 0 and 0 <= rank < world")
    per = -(-total // world)
    start = min(rank * per, total)
    return start, min(start + per, total)


def shard_prompts(prompts: np.ndarray, world: int, rank: int) -> np.ndarray:
    """Columns (requests) of a ``[context, requests]`` prompt matrix owned by ``rank``."""
    start, stop = request_range(prompts.shape[1], world, rank)
    return np.ascontiguousarray(prompts[:, start:stop])
