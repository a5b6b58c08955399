"""A save that hashes only the blocks it has not seen (DigestCache), on a B200, against the oracle.

Every digest a save returns must equal the oracle's SHA-256 and CRC32C of the
packed block, whether it was computed or served from the cache:
* a second save of the same blocks under the same generations is served for
  every full block;
* a block the engine changed without a new generation (a caller error) is
  caught by its CRC32C, counted as rejected, and hashed after all;
* a restore records the snapshot's digests for the blocks it wrote, so saving
  those blocks next is served too.
"""
import pytest
import torch

from cases import golden_case
from gpu_cases import cuda_5d
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_saves_hash_only_unseen_blocks():
    from kvsnap_b200.dataplane import DigestCache, PendingDigests, TorchBlockDataPlane
    case, storages, layout = golden_case("qwen3_8b_5d")
    _, tensors, caches = cuda_5d(case)
    plane = TorchBlockDataPlane(caches, 16, 256 << 20)
    try:
        size = plane.block_bytes
        saved = list(case["saved"])
        tokens = len(saved) * 16 - 3                          # a partial last block: never cached
        generations = [1] * len(saved)
        cache = DigestCache()
        snap = plane.pool.reserve(len(saved) * size)
        targets = [(snap, i * size) for i in range(len(saved))]

        want = oracle.digests(oracle.pack(storages, layout, saved, tokens))
        cold, warm = [], []
        plane.save_gather(saved, targets, tokens, digests=cold, cache=cache, generations=generations)
        assert [tuple(d) for d in cold] == want
        assert cache.hits == 0 and cache.misses == len(saved) - 1 and len(cache) == len(saved) - 1
        plane.save_gather(saved, targets, tokens, digests=warm, cache=cache, generations=generations)
        assert [tuple(d) for d in warm] == want
        assert cache.hits == len(saved) - 1 and cache.rejected == 0

        # The engine changes block saved[1] but the caller keeps its generation: its CRC gives it away.
        layer = next(iter(tensors))
        flat = tensors[layer]
        block_bytes_in_layer = flat.numel() // 2 // case["num_blocks"]
        at = saved[1] * block_bytes_in_layer + 77                 # K half of that layer, block saved[1]
        flat[at] = flat[at] ^ 0x55
        storages[layer][at] ^= 0x55
        pending = PendingDigests()
        plane.save_gather(saved, targets, tokens, digests=pending, cache=cache, generations=generations)
        got = pending.result()
        assert [tuple(d) for d in got] == oracle.digests(oracle.pack(storages, layout, saved, tokens))
        assert cache.rejected == 1

        # A restore records the snapshot's digests for the blocks it writes.
        restored = [b for b in range(case["num_blocks"]) if b not in saved][: len(saved)]
        new_generations = [7] * (len(saved) - 1) + [None]     # the partial last block stays unrecorded
        plane.load_scatter(restored, targets, cache=cache, generations=new_generations,
                           known_digests=[tuple(d) for d in got])
        hits = cache.hits
        again = []
        plane.save_gather(restored, targets, tokens, digests=again, cache=cache, generations=new_generations[:-1] + [8])
        assert [tuple(d) for d in again] == [tuple(d) for d in got]
        assert cache.hits == hits + len(saved) - 1
        snap.close()
    finally:
        plane.close()


def test_cache_arguments_are_checked():
    from kvsnap_b200.dataplane import DigestCache, TorchBlockDataPlane
    case, storages, layout = golden_case("qwen3_8b_5d")
    _, tensors, caches = cuda_5d(case)
    plane = TorchBlockDataPlane(caches, 16, 64 << 20)
    try:
        snap = plane.pool.reserve(2 * plane.block_bytes)
        targets = [(snap, 0), (snap, plane.block_bytes)]
        with pytest.raises(ValueError, match="generation"):
            plane.save_gather([1, 2], targets, 32, digests=[], cache=DigestCache())
        with pytest.raises(ValueError, match="digests"):
            plane.save_gather([1, 2], targets, 32, cache=DigestCache(), generations=[0, 0])
        with pytest.raises(ValueError, match="known digest"):
            plane.load_scatter([1, 2], targets, cache=DigestCache(), generations=[0, 0])
        snap.close()
    finally:
        plane.close()
