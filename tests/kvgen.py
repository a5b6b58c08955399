"""Deterministic synthetic KV bytes and block tables shared by the tests, fixtures and bench.

A splitmix64 stream keyed by (seed, index) gives the same bytes on every
machine and numpy version, so golden fixtures can store a seed instead of the
cache contents. Values are raw 16-bit patterns, NaNs included, as the
reference's own data-plane tests use (they compare bits, never values).
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


_MIX1, _MIX2 = 0xBF58476D1CE4E5B9, 0x94D049BB133111EB


def random_words(seed: int, first: int, count: int) -> np.ndarray:
    """Words ``first .. first+count-1`` of the splitmix64 stream keyed by ``seed``."""
    with np.errstate(over="ignore"):
        z = np.arange(first, first + count, dtype=np.uint64) + np.uint64(seed) * _GOLDEN + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(_MIX1)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(_MIX2)
        return z ^ (z >> np.uint64(31))


def random_bytes(seed: int, nbytes: int) -> np.ndarray:
    """``nbytes`` pseudo-random bytes: splitmix64 of (seed, word index), little-endian."""
    return random_words(seed, 0, (nbytes + 7) // 8).view(np.uint8)[:nbytes].copy()


class LazyBytes:
    """``random_bytes(seed, nbytes)`` as a read-only buffer that generates only the slices read.

    Stands in for a whole cache layer in the oracle's ``storages`` at sizes
    (gigabytes a layer) where materialising the layer on the host is not worth it:
    ``oracle.pack`` only slices its storages.
    """

    def __init__(self, seed: int, nbytes: int):
        self.seed, self.nbytes = seed, nbytes

    def __len__(self):
        return self.nbytes

    def __getitem__(self, key):
        if not isinstance(key, slice) or key.step not in (None, 1):
            raise TypeError("LazyBytes takes contiguous slices")
        start, stop, _ = key.indices(self.nbytes)
        if stop <= start:
            return np.empty(0, dtype=np.uint8)
        first = start // 8
        words = random_words(self.seed, first, (stop + 7) // 8 - first)
        return words.view(np.uint8)[start - 8 * first:stop - 8 * first]


def fill_random(buffer, seed: int, chunk_words: int = 1 << 26) -> None:
    """Fill a contiguous torch uint8 tensor (any device; size a multiple of 8) with ``random_bytes(seed, len)``.

    The same splitmix64 stream in int64 torch arithmetic (wrapping multiplies,
    logical shifts by masking), so a cache of many gigabytes is filled on the GPU
    and the oracle regenerates any part of it on the host.
    """
    import torch
    words = buffer.view(torch.int64)
    signed = lambda v: v - (1 << 64) if v >= 1 << 63 else v   # noqa: E731
    start = signed((seed * int(_GOLDEN) + int(_GOLDEN)) % (1 << 64))
    mix1, mix2 = signed(_MIX1), signed(_MIX2)

    def lsr(z, k):
        return (z >> k) & ((1 << (64 - k)) - 1)

    for first in range(0, words.numel(), chunk_words):
        count = min(chunk_words, words.numel() - first)
        z = torch.arange(first, first + count, dtype=torch.int64, device=buffer.device) + start
        z = (z ^ lsr(z, 30)) * mix1
        z = (z ^ lsr(z, 27)) * mix2
        words[first:first + count] = z ^ lsr(z, 31)


def permutation(seed: int, n: int) -> list:
    """A seeded permutation of range(n) (numpy PCG64, stable across numpy versions)."""
    return [int(v) for v in np.random.Generator(np.random.PCG64(seed)).permutation(n)]


def disjoint_block_sets(seed: int, num_blocks: int, count: int) -> tuple:
    """Two disjoint lists of ``count`` block ids from 1..num_blocks-1 (block 0 is vLLM's null block)."""
    order = [b + 1 for b in permutation(seed, num_blocks - 1)]
    return order[:count], order[count:2 * count]
