"""Parity at the benchmark configurations' full sizes, on a B200, against the CPU oracle.

The caches here are the sizes the benchmark configurations name (7 GiB for the
Qwen3-1.7B plumbing case, up to 30 GiB for the rotation), so they are filled on
the GPU with the splitmix64 stream of ``kvgen`` and the oracle regenerates on
the host exactly the byte ranges it reads (``kvgen.LazyBytes``): the checks are
the oracle's, byte for byte, with no copy of a whole cache to the host.

* Save and restore at full size, every packed byte against ``oracle.pack``,
  every content id and CRC32C against ``hashlib`` and the oracle's CRC, and the
  whole cache after the restore against ``oracle.unpack``: benchmark
  configuration 1 (28 layers x 4096 blocks, a 128-block session from a seeded
  permutation of 1..4095, restored into a disjoint set) in both save and restore
  modes; layers of more than 4 GiB (Qwen3-32B TP-1 geometry, 70000 blocks) with
  block ids at the top of the pool, so that every cache offset of the V half
  needs 64-bit arithmetic; and Qwen3-32B TP-4 and TP-8 shards.
* Benchmark configuration 3: 512- and 2048-block Qwen3-8B restores from a
  pinned staging buffer with seeded corruption of 1 block in 1000 (at least
  one), which must flag exactly those blocks and leave the cache untouched
  (reference kvsnap/store/store.py:686-723 checks each block on the host).
* Benchmark configuration 4: 64 sessions of log-uniform length, the second 32
  forking the first 32 with 75 % of their blocks copied, saved through the API:
  every GPU content id equals ``hashlib`` of the saved bytes, and the dedup rate
  equals the oracle's (kvsnap/store/store.py:625-628, connector/volatile.py:254-279).
"""
import ctypes as C
import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

import kvgen
from oracle import oracle

pytestmark = pytest.mark.gpu

HEAD_DIM, BLOCK = 128, 16


class FormulaCache:
    """Per layer a ``[2, blocks, 16, heads, 128]`` bf16 CUDA cache holding ``kvgen.random_bytes(seed * 1000 + i)``,
    and the oracle's view of the same bytes (lazy storages, the 5-D layer split in name order)."""

    def __init__(self, seed, layers, blocks, heads):
        self.raw, self.caches, self.storages, views = {}, {}, {}, {}
        per_layer = 2 * blocks * BLOCK * heads * HEAD_DIM * 2
        for i in range(layers):
            name = f"model.layers.{i}"
            buf = torch.empty(per_layer, dtype=torch.uint8, device="cuda")
            kvgen.fill_random(buf, seed * 1000 + i)
            self.raw[name] = buf
            self.caches[name] = buf.view(torch.bfloat16).view(2, blocks, BLOCK, heads, HEAD_DIM)
            self.storages[name] = kvgen.LazyBytes(seed * 1000 + i, per_layer)
            views.update(oracle.split_5d(name, name, 0, blocks, BLOCK, heads, HEAD_DIM, 2))
        self.layout = oracle.register(views, BLOCK)

    def rows(self, raw, span):
        """Span ``span`` of every cache block as a ``[blocks, span bytes]`` view of its layer's bytes."""
        return raw[span.storage].as_strided((span.blocks, span.bytes), (span.pitch, 1), span.start)

    def unpack_into(self, raw, block_ids, packed_rows):
        """``oracle.unpack`` applied on the GPU: every span of the oracle's layout, rows ``block_ids``,
        takes that span's bytes of each packed block (``packed_rows``: ``[n, block_bytes]`` CUDA uint8)."""
        ids = torch.tensor(block_ids, dtype=torch.int64, device="cuda")
        for span in self.layout.spans:
            self.rows(raw, span)[ids] = packed_rows[:, span.offset:span.offset + span.bytes]


def pinned(allocation, offset=0, size=None):
    """A numpy view of pinned pool memory (no copy)."""
    size = allocation.size - offset if size is None else size
    return np.ctypeslib.as_array((C.c_uint8 * size).from_address(allocation.pointer + offset))


def host_checksums(buffers, sha=True):
    """``(hashlib content id, oracle CRC32C)`` of each buffer, on the host's cores (both release the GIL)."""
    oracle.crc32c(b"")                       # builds the oracle's table before the threads share it
    work = (lambda b: (oracle.sha256_hex(b), oracle.crc32c(b))) if sha else oracle.crc32c
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        return list(pool.map(work, buffers))


def release(plane, cache):
    """Close the plane and hand the cache's memory back, so the next full-size case finds the GPU empty
    even when this one failed (a failed test's frame keeps its locals alive)."""
    plane.close()
    plane.caches.clear()
    for table in (cache.raw, cache.caches, cache.storages):
        table.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


GEOMETRIES = {
    # benchmark configuration 1 at its size; a full last block, then a partial one through the direct kernels
    "config1-staged": dict(layers=28, heads=8, blocks=4096, n=128, tokens=2048, save="staged", restore="staged"),
    "config1-direct-tail": dict(layers=28, heads=8, blocks=4096, n=128, tokens=2043, save="direct",
                                restore="direct"),
    # per-layer tensors of 4.6 GB, block ids in the top 256 of the pool
    "tp1-4gib-layers-top-ids": dict(layers=2, heads=8, blocks=70000, n=64, tokens=64 * 16 - 7, save="staged",
                                    restore="staged", top=True),
    # Qwen3-32B shards: 64 layers of 8 KiB (TP-4, runs) and 4 KiB (TP-8, runs of pairs) spans
    "tp4-shard": dict(layers=64, heads=2, blocks=4096, n=512, tokens=8192, save="staged", restore="staged"),
    "tp8-shard-tail": dict(layers=64, heads=1, blocks=4096, n=512, tokens=8192 - 3, save="staged",
                           restore="staged"),
}


@pytest.mark.parametrize("geometry", list(GEOMETRIES))
def test_full_size_save_and_restore_match_the_oracle(geometry):
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    g = GEOMETRIES[geometry]
    n, blocks = g["n"], g["blocks"]
    cache = FormulaCache(11, g["layers"], blocks, g["heads"])
    if g.get("top"):
        order = [blocks - 256 + b for b in kvgen.permutation(5, 256)]
        saved, restored = order[:n], order[n:2 * n]
    else:
        saved, restored = kvgen.disjoint_block_sets(17, blocks, n)
    size = cache.layout.block_bytes
    plane = TorchBlockDataPlane(cache.caches, BLOCK, n * size + (64 << 20), save_mode=g["save"],
                                restore_mode=g["restore"])
    try:
        plane.warm_up()
        assert plane.block_bytes == size
        assert [layer["name"] for layer in plane.layers] == [s.name for s in cache.layout.spans]
        snapshot = plane.pool.reserve(n * size)
        targets = [(snapshot, i * size) for i in range(n)]
        digests = [] if g["save"] == "staged" else None
        plane.save_gather(saved, targets, g["tokens"], digests=digests)

        expected = oracle.pack(cache.storages, cache.layout, saved, g["tokens"])
        got = pinned(snapshot)
        for i, block in enumerate(expected):
            assert np.array_equal(got[i * size:(i + 1) * size], block), f"packed block {i}"
        if digests is None:                  # the direct save returns no digests: hash the pinned blocks on the GPU
            digests = plane.digest(targets)
        assert [tuple(d) for d in digests] == host_checksums(expected)

        before = {k: v.clone() for k, v in cache.raw.items()}
        progress = []
        plane.load_scatter(restored, targets, progress=progress)
        assert [left for _, left in progress] == oracle.progress_lefts(n, size)
        cache.unpack_into(before, restored, torch.from_numpy(np.stack(expected)).cuda())
        torch.cuda.synchronize()
        for name in cache.raw:
            assert torch.equal(cache.raw[name], before[name]), f"{name} after the restore"
        snapshot.close()
    finally:
        release(plane, cache)


@pytest.mark.parametrize("n", [512, 2048])
def test_disk_tier_restore_flags_exactly_the_corrupted_blocks(n):
    """Benchmark configuration 3: 8k / 32k-token Qwen3-8B restores from pinned staging, 1 block in 1000 corrupt."""
    from kvsnap_b200.dataplane import CorruptBlockError, TorchBlockDataPlane
    pool_blocks = 4096
    cache = FormulaCache(31, 36, pool_blocks, 8)
    size = cache.layout.block_bytes
    plane = TorchBlockDataPlane(cache.caches, BLOCK, n * size + (64 << 20))
    try:
        plane.warm_up()
        staging = plane.pool.reserve(n * size)
        host = pinned(staging)
        payload = torch.empty(n * size, dtype=torch.uint8, device="cuda")   # the blocks the readers brought in
        kvgen.fill_random(payload, 9000 + n)
        torch.from_numpy(host).copy_(payload)
        sources = [(staging, i * size) for i in range(n)]
        crcs = host_checksums([host[i * size:(i + 1) * size] for i in range(n)], sha=False)
        ids = [b + 1 for b in kvgen.permutation(70 + n, pool_blocks - 1)[:n]]    # freshly allocated, fragmented
        rng = np.random.Generator(np.random.PCG64(n))
        bad = [i for i in range(n) if rng.random() < 1 / 1000] or [int(rng.integers(n))]
        flips = {i: i * size + int(rng.integers(size)) for i in bad}
        for at in flips.values():
            host[at] ^= 0x5A
        id_t = torch.tensor(ids, dtype=torch.int64, device="cuda")
        # Compared as 16-bit patterns: random bf16 bits hold NaNs, which never compare equal as values.
        bits = {name: t.view(torch.int16) for name, t in cache.caches.items()}
        before = {name: b[:, id_t].clone() for name, b in bits.items()}
        progress = []
        with pytest.raises(CorruptBlockError) as err:
            plane.load_scatter(ids, sources, progress=progress, expected_crc32c=crcs)
        assert err.value.blocks == bad
        assert progress == []
        for name, b in bits.items():
            assert torch.equal(b[:, id_t], before[name]), f"{name} changed by a rejected restore"
        del before
        for at in flips.values():
            host[at] ^= 0x5A
        per_launch = (64 << 20) // size
        assert plane.load_scatter(ids, sources, expected_crc32c=crcs) == math.ceil(n / per_launch)
        payload.copy_(torch.from_numpy(host))
        for span in cache.layout.spans:
            assert torch.equal(cache.rows(cache.raw, span)[id_t], payload.view(n, size)[:, span.offset:
                                                                                    span.offset + span.bytes])
        staging.close()
    finally:
        release(plane, cache)


def test_rotation_dedup_rate_matches_the_oracle():
    """Benchmark configuration 4: 64 Qwen3-1.7B sessions, forks sharing 75 % of their parents' blocks."""
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    pool_blocks = 16384
    rng = np.random.Generator(np.random.PCG64(44))
    lengths = np.exp(rng.uniform(np.log(512), np.log(8192), 64)).astype(int)
    for child in range(32, 64):                          # a fork is at least as long as its parent
        lengths[child] = max(lengths[child], lengths[child - 32])
    free = [int(b) + 1 for b in rng.permutation(pool_blocks - 1)]
    sessions = [(int(t), [free.pop() for _ in range((int(t) + BLOCK - 1) // BLOCK)]) for t in lengths]
    cache = FormulaCache(44, 28, pool_blocks, 8)
    for child in range(32, 64):                          # forks copy 75 % of the parent's full blocks
        parent = sessions[child - 32][1]
        shared = (len(parent) - 1) * 3 // 4
        src = torch.tensor(parent[:shared], device="cuda")
        dst = torch.tensor(sessions[child][1][:shared], device="cuda")
        for t in cache.caches.values():
            bits = t.view(torch.int16)
            bits[:, dst] = bits[:, src]
    size = cache.layout.block_bytes
    plane = TorchBlockDataPlane(cache.caches, BLOCK, max(len(b) for _, b in sessions) * (size + 16) + (64 << 20))
    try:
        plane.warm_up()
        gpu, host, lengths_all = [], [], []
        for tokens, blocks in sessions:
            owned = [plane.pool.reserve(size) for _ in blocks]          # one allocation a block, as the host tier
            digests = []
            plane.save_gather(blocks, [(a, 0) for a in owned], tokens, digests=digests)
            mine = host_checksums([pinned(a) for a in owned])
            assert [tuple(d) for d in digests] == mine
            gpu += [d[0] for d in digests]
            host += mine
            lengths_all += [size] * len(blocks)
            for a in owned:
                a.close()
        unique, segments = oracle.dedup_digests(host, lengths_all)
        oracle_rate = 1 - len(unique) / len(segments)
        gpu_rate = 1 - len(set(gpu)) / len(gpu)
        assert [s["blob_id"] for s in segments] == gpu
        assert gpu_rate == oracle_rate
        assert gpu_rate > 0.2                                         # the forks' shared blocks deduplicate
    finally:
        release(plane, cache)
