"""Deterministic synthetic KV bytes and block tables shared by the tests, fixtures and bench.

A splitmix64 stream keyed by (seed, index) gives the same bytes on every
machine and numpy version, so golden fixtures can store a seed instead of the
cache contents. Values are raw 16-bit patterns, NaNs included, as the
reference's own data-plane tests use (they compare bits, never values).
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def random_bytes(seed: int, nbytes: int) -> np.ndarray:
    """``nbytes`` pseudo-random bytes: splitmix64 of (seed, word index), little-endian."""
    words = (nbytes + 7) // 8
    with np.errstate(over="ignore"):
        z = np.arange(words, dtype=np.uint64) + np.uint64(seed) * _GOLDEN + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z.view(np.uint8)[:nbytes].copy()


def permutation(seed: int, n: int) -> list:
    """A seeded permutation of range(n) (numpy PCG64, stable across numpy versions)."""
    return [int(v) for v in np.random.Generator(np.random.PCG64(seed)).permutation(n)]


def disjoint_block_sets(seed: int, num_blocks: int, count: int) -> tuple:
    """Two disjoint lists of ``count`` block ids from 1..num_blocks-1 (block 0 is vLLM's null block)."""
    order = [b + 1 for b in permutation(seed, num_blocks - 1)]
    return order[:count], order[count:2 * count]
