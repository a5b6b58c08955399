"""Device staging stays within ``staging_bytes``, on a B200, with results identical to the oracle's.

A serving worker's KV cache takes most of the GPU, so a save or a verified
restore may only stage through a bounded amount of device memory (the
reference stages one 64 MiB chunk, kvsnap/connector/dataplane.py:409-417).
A Qwen3-8B session of 512 blocks (1.2 GB packed) is saved through a 256 MiB
bound: peak device memory grows by at most the bound plus the block tables,
the packed bytes are the oracle's, and the content ids and CRC32Cs equal
``hashlib`` and the oracle's CRC, with and without a digest cache serving some
blocks. A verified restore above the bound checks every block before any KV
write and keeps to its two-chunk ring; ``digest`` above the bound hashes the
pinned blocks in place. SHA-256 in parts (``kvsnap_dp_sha256_part``) equals
``hashlib`` for part cuts at every chunk position.
"""
import ctypes as C
import hashlib
import random

import numpy as np
import pytest
import torch

import kvgen
from oracle import oracle
from test_gpu_full_size import FormulaCache, host_checksums, pinned, release

pytestmark = pytest.mark.gpu

BOUND = 256 << 20


def _growth(fn):
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    before = torch.cuda.memory_allocated()
    result = fn()
    torch.cuda.synchronize()
    return result, torch.cuda.max_memory_allocated() - before


@pytest.mark.parametrize("tokens", [8192, 8192 - 9])
def test_save_and_verified_restore_stay_within_the_staging_bound(tokens):
    from kvsnap_b200.dataplane import CorruptBlockError, DigestCache, PendingDigests, TorchBlockDataPlane
    n, pool_blocks = 512, 1100
    cache = FormulaCache(23, 36, pool_blocks, 8)
    size = cache.layout.block_bytes
    saved, restored = kvgen.disjoint_block_sets(29, pool_blocks, n)
    plane = TorchBlockDataPlane(cache.caches, 16, 2 * n * (size + 16) + (64 << 20), staging_bytes=BOUND)
    try:
        plane.warm_up()
        assert n * size > BOUND
        snapshot = plane.pool.reserve(n * size)
        targets = [(snapshot, i * size) for i in range(n)]
        digests = []
        _, grew = _growth(lambda: plane.save_gather(saved, targets, tokens, digests=digests))
        assert grew <= BOUND + (8 << 20), f"save staged {grew} bytes of device memory"
        expected = oracle.pack(cache.storages, cache.layout, saved, tokens)
        got = pinned(snapshot)
        for i, block in enumerate(expected):
            assert np.array_equal(got[i * size:(i + 1) * size], block), f"packed block {i}"
        want = host_checksums(expected)
        assert [tuple(d) for d in digests] == want

        # Per-block targets (the host tier's), a pending result and a digest cache that knows half the blocks.
        owned = [plane.pool.reserve(size) for _ in range(n)]
        digest_cache, generations = DigestCache(), list(range(n))
        for i in range(0, n - 1, 2):
            digest_cache.put(saved[i], generations[i], want[i])
        pending = PendingDigests()
        plane.save_gather(saved, [(a, 0) for a in owned], tokens, digests=pending, cache=digest_cache,
                          generations=generations)
        assert [tuple(d) for d in pending.result()] == want
        assert digest_cache.hits == len(range(0, n - 1, 2)) and digest_cache.rejected == 0
        for i, a in enumerate(owned):
            assert np.array_equal(pinned(a), expected[i]), f"per-block target {i}"
        # Columns landed by the copy engine: per-block targets at one pitch (one transfer a column), then
        # the same allocations in shuffled order, where no one pitch spaces them and the kernel lands them.
        plane.column_landing = "copy"
        from kvsnap_b200.dataplane import _even_pitch
        assert _even_pitch([a.pointer for a in owned], 0, n, size) is not None   # reserved back to back
        for targets_now in (list(owned), random.Random(5).sample(owned, n)):
            for a in owned:
                C.memset(a.pointer, 0, size)
            got_digests = []
            plane.save_gather(saved, [(a, 0) for a in targets_now], tokens, digests=got_digests)
            assert [tuple(d) for d in got_digests] == want
            for i, a in enumerate(targets_now):
                assert np.array_equal(pinned(a), expected[i]), f"copy-engine landing, target {i}"
        plane.column_landing = "kernel"

        crcs = [c for _, c in want]
        bits = {name: t.view(torch.int16) for name, t in cache.caches.items()}
        ids = torch.tensor(restored, dtype=torch.int64, device="cuda")
        before = {name: b[:, ids].clone() for name, b in bits.items()}
        flip = snapshot.pointer + 7 * size + 4242
        C.memset(flip, C.string_at(flip, 1)[0] ^ 0x21, 1)
        with pytest.raises(CorruptBlockError) as err:
            plane.load_scatter(restored, targets, expected_crc32c=crcs)
        assert err.value.blocks == [7]
        for name, b in bits.items():
            assert torch.equal(b[:, ids], before[name]), f"{name} changed by a rejected restore"
        C.memset(flip, C.string_at(flip, 1)[0] ^ 0x21, 1)
        progress = []
        _, grew = _growth(lambda: plane.load_scatter(restored, targets, expected_crc32c=crcs, progress=progress))
        assert grew <= 2 * (64 << 20) + (8 << 20), f"verified restore staged {grew} bytes"
        assert [left for _, left in progress] == oracle.progress_lefts(n, size)
        packed = torch.from_numpy(np.stack(expected)).cuda()
        for span in cache.layout.spans:
            assert torch.equal(cache.rows(cache.raw, span)[ids], packed[:, span.offset:span.offset + span.bytes])

        result, grew = _growth(lambda: plane.digest(targets))
        assert grew <= 8 << 20
        assert [tuple(d) for d in result] == want
        snapshot.close()
        for a in owned:
            a.close()
    finally:
        release(plane, cache)


@pytest.mark.parametrize("length", [64, 1000, 4096 + 48, 65536 + 8, 2359296])
def test_sha256_in_parts_matches_hashlib(length):
    from kvsnap_b200.dataplane import _dp, _load
    lib = _dp(_load())
    n = 33
    data = [kvgen.random_bytes(7000 + length + i, length) for i in range(n)]
    stride = (length + 15) // 16 * 16
    host = np.zeros(n * stride, dtype=np.uint8)
    for i, d in enumerate(data):
        host[i * stride:i * stride + length] = d
    buf = torch.from_numpy(host).cuda()
    state = torch.empty(n * 8, dtype=torch.int32, device="cuda")
    out = torch.empty(n * 32, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    chunks = length // 64
    cuts = sorted({0, length} | {64 * c for c in (1, chunks // 3, chunks // 2, chunks - 1) if 0 < c < chunks})
    for a, b in zip(cuts, cuts[1:]):
        addrs = torch.tensor([buf.data_ptr() + i * stride + a for i in range(n)], dtype=torch.int64, device="cuda")
        last = b == length
        assert lib.kvsnap_dp_sha256_part(addrs.data_ptr(), n, b - a, a, length, state.data_ptr(),
                                         out.data_ptr() if last else 0, stream) == 0
        torch.cuda.synchronize()
    got = out.cpu().numpy().tobytes()
    assert [got[32 * i:32 * i + 32].hex() for i in range(n)] == [hashlib.sha256(d.tobytes()).hexdigest() for d in data]
    # A part before the last must be whole chunks, and a later part needs the state.
    addrs = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    if length > 64:
        assert lib.kvsnap_dp_sha256_part(addrs.data_ptr(), 1, 63, 0, length, state.data_ptr(), 0, stream) == -1
        assert lib.kvsnap_dp_sha256_part(addrs.data_ptr(), 1, length - 64, 64, length, 0, out.data_ptr(),
                                         stream) == -1


def test_landing_kernel_stores_columns_at_their_targets():
    """kvsnap_dp_land: column bytes of each block to target + offset, in pinned and device memory; a
    misaligned target is flagged and skipped, the others still land."""
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import CudaPool, _dp
    pool = CudaPool(4 << 20, 0)
    lib = _dp(pool.lib)
    try:
        n, stride, length, offset = 5, 12288, 10000 // 16 * 16, 4096 + 32
        src = torch.from_numpy(kvgen.random_bytes(3, n * stride)).cuda()
        host = pool.reserve(n * 32768 + 16)
        device = torch.zeros(n * 32768, dtype=torch.uint8, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        for base, view in ((host.pointer, lambda: pinned(host)[:n * 32768]), (device.data_ptr(), lambda: device.cpu().numpy())):
            places = [base + ((i * 3) % n) * 32768 for i in range(n)]
            places[2] += 8 if base == host.pointer else 0                  # a misaligned target in the pinned case
            targets = torch.tensor(places, dtype=torch.int64, device="cuda")
            assert lib.kvsnap_dp_land(src.data_ptr(), stride, targets.data_ptr(), offset, n, length,
                                      status.data_ptr(), 0, stream) == 0
            torch.cuda.synchronize()
            got, want = view(), src.cpu().numpy()
            for i in range(n):
                at = places[i] - base + offset
                if places[i] % 16:
                    assert int(status.item()) & _abi.MISALIGNED
                    continue
                assert np.array_equal(got[at:at + length], want[i * stride:i * stride + length]), i
        assert lib.kvsnap_dp_land(src.data_ptr(), 8, targets.data_ptr(), 0, n, 16, status.data_ptr(), 0, stream) == -1
        host.close()
    finally:
        pool.close()


def test_strided_landing_moves_a_column_to_evenly_spaced_targets():
    """kvsnap_dp_land_strided: row i of a device column (src + i * stride) to dst + i * pitch in pinned
    memory, one copy-engine transfer; rows that would overlap are refused."""
    from kvsnap_b200.dataplane import CudaPool, _dp
    pool = CudaPool(4 << 20, 0)
    lib = _dp(pool.lib)
    try:
        n, stride, length, pitch, offset = 7, 12288, 10000, 32768 + 48, 4096 + 8
        src = torch.from_numpy(kvgen.random_bytes(4, n * stride)).cuda()
        host = pool.reserve(n * pitch + offset)
        C.memset(host.pointer, 0xA5, n * pitch + offset)
        stream = torch.cuda.current_stream().cuda_stream
        assert lib.kvsnap_dp_land_strided(src.data_ptr(), stride, host.pointer + offset, pitch, n, length, stream) == 0
        torch.cuda.synchronize()
        got, want = pinned(host), src.cpu().numpy()
        for i in range(n):
            at = offset + i * pitch
            assert np.array_equal(got[at:at + length], want[i * stride:i * stride + length]), i
            assert (got[at + length:at + pitch] == 0xA5).all(), f"row {i} wrote past its length"
        assert (got[:offset] == 0xA5).all()
        assert lib.kvsnap_dp_land_strided(src.data_ptr(), stride, host.pointer, length - 1, n, length, stream) == -1
        assert lib.kvsnap_dp_land_strided(src.data_ptr(), length - 16, host.pointer, pitch, n, length, stream) == -1
        assert lib.kvsnap_dp_land_strided(src.data_ptr(), stride, host.pointer, pitch, 0, length, stream) == 0
        host.close()
    finally:
        pool.close()


def test_concurrent_bounded_saves_keep_their_own_digests():
    """Two save threads at once through the bounded path, as the connector's two save workers run
    (kvsnap/connector/vllm.py:202): every save's hash state and outputs stay its own until its digests
    are read, so the packed bytes and content ids of each equal the oracle's."""
    from concurrent.futures import ThreadPoolExecutor
    from kvsnap_b200.dataplane import PendingDigests, TorchBlockDataPlane
    n, pool_blocks, sessions = 160, 1100, 6
    cache = FormulaCache(37, 36, pool_blocks, 8)
    size = cache.layout.block_bytes
    order = [b + 1 for b in kvgen.permutation(41, pool_blocks - 1)]
    block_sets = [order[k * n:(k + 1) * n] for k in range(sessions)]
    plane = TorchBlockDataPlane(cache.caches, 16, sessions * n * (size + 16) + (64 << 20), staging_bytes=BOUND)
    try:
        plane.warm_up()
        assert n * size > BOUND
        owned = [[plane.pool.reserve(size) for _ in range(n)] for _ in range(sessions)]

        def save(k):
            pending = PendingDigests()
            plane.save_gather(block_sets[k], [(a, 0) for a in owned[k]], n * 16 - 3 * (k % 2), digests=pending)
            return pending.result()

        with ThreadPoolExecutor(max_workers=2) as savers:
            results = list(savers.map(save, range(sessions)))
        for k in range(sessions):
            expected = oracle.pack(cache.storages, cache.layout, block_sets[k], n * 16 - 3 * (k % 2))
            for i, a in enumerate(owned[k]):
                assert np.array_equal(pinned(a), expected[i]), f"session {k} block {i}"
            assert [tuple(d) for d in results[k]] == host_checksums(expected), f"session {k}"
        for blocks in owned:
            for a in blocks:
                a.close()
    finally:
        release(plane, cache)
