"""Batch sharding of independent environments across ranks (one process per GPU).

Environments never exchange data on the inference path, so N GPUs each run a
contiguous slice of the batch with replicated weights and no collective. The
inputs of environment g are generated from (seed, g) alone, so a shard's rows
equal the same rows of a one-process run byte for byte.
"""
from __future__ import annotations

import numpy as np


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the environments owned by `rank` (contiguous, sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def env_planes(seed: int, env: int, seq: int, planes: int = 3, dim: int = 128) -> np.ndarray:
    """fp16 U(0,1) input planes [seq][planes][dim][dim] of one environment."""
    rng = np.random.default_rng([seed, env])
    return rng.random(size=(seq, planes, dim, dim), dtype=np.float32).astype(np.float16)


def shard_planes(seed: int, start: int, stop: int, seq: int, planes: int = 3, dim: int = 128) -> np.ndarray:
    """Rows b*seq + t of environments [start, stop)."""
    return np.concatenate([env_planes(seed, e, seq, planes, dim) for e in range(start, stop)], axis=0)
