"""Sharding of independent utterances across GPUs (no collective on the
data path: each rank runs its own queue).

The pool of P utterances is dealt round-robin into P / B interleaved blocks
of B utterances (block b = {b, b + P/B, b + 2P/B, ...}); at step k rank r of
N processes block (r + N k) mod (P / B). Every rank thus runs a batch of B
distinct utterances per step (weak scaling); with N * B <= P the ranks'
batches of one step are disjoint, beyond that blocks repeat across ranks.
"""
from __future__ import annotations

from math import gcd
from typing import List


def n_blocks(pool_size: int, batch: int) -> int:
    if pool_size % batch:
        raise ValueError("pool size must be a multiple of the batch")
    return pool_size // batch


def block(pool_size: int, batch: int, b: int) -> List[int]:
    nb = n_blocks(pool_size, batch)
    return [b + nb * j for j in range(batch)]


def rank_batch(pool_size: int, rank: int, world: int, batch: int, step: int) -> List[int]:
    nb = n_blocks(pool_size, batch)
    return block(pool_size, batch, (rank + world * step) % nb)


def period(pool_size: int, world: int, batch: int) -> int:
    """Number of distinct batches a rank cycles through."""
    nb = n_blocks(pool_size, batch)
    return nb // gcd(nb, world % nb) if world % nb else 1


def rank_batches(pool_size: int, rank: int, world: int, batch: int) -> List[List[int]]:
    return [rank_batch(pool_size, rank, world, batch, k) for k in range(period(pool_size, world, batch))]
