"""Parity of the CUDA data plane with the reference, on a B200.

Every case feeds the CUDA path and the CPU oracle (oracle/oracle.py) the same
seeded bytes and requires identical results: packed blocks byte for byte,
CRC32C and SHA-256 digests equal to the golden values the reference itself
produced (tests/golden/golden.json), the KV cache bit-exact after a restore,
and the reference's copy counts, launch counts and progress lists.
"""
import ctypes as C
import hashlib
import random

import numpy as np
import pytest
import torch

import kvgen
from cases import GOLDEN, golden_case, sha_of, storages_small
from gpu_cases import cuda_5d, cuda_small, cuda_vllm031, host_bytes
from oracle import oracle

pytestmark = pytest.mark.gpu

LARGE = ["vllm031", "qwen3_1p7b_5d", "qwen3_8b_5d"]


def plane_for(caches, block_size=16, **kwargs):
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    plane = TorchBlockDataPlane(caches, block_size, 256 << 20, **kwargs)
    plane.warm_up()
    return plane


def cuda_case(key):
    case, storages, layout = golden_case(key)
    build = cuda_5d if case["kind"] == "5d" else cuda_vllm031
    _, tensors, caches = build(case)
    return case, storages, layout, tensors, caches


def targets_for(plane, kind, count):
    size = plane.block_bytes
    if kind == "per-block":
        owned = [plane.pool.reserve(size) for _ in range(count)]
        return owned, [(a, 0) for a in owned]
    staged = plane.pool.reserve(size * count)
    return [staged], [(staged, i * size) for i in range(count)]


@pytest.mark.parametrize("key", LARGE)
@pytest.mark.parametrize("save_mode", ["staged", "direct"])
def test_save_gather_packs_like_the_reference(key, save_mode):
    case, storages, layout, tensors, caches = cuda_case(key)
    plane = plane_for(caches, save_mode=save_mode)
    try:
        assert plane.layers == case["layers"]
        assert plane.block_bytes == case["block_bytes"]
        expected = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        n, size = len(case["saved"]), plane.block_bytes
        for kind in ("per-block", "staging"):
            for chunk in (64 << 20, int(case["restore_chunk_bytes"])):
                owned, targets = targets_for(plane, kind, n)
                digests = [] if save_mode == "staged" else None
                copies = plane.save_gather(case["saved"], targets, case["num_kv_tokens"], chunk_bytes=chunk,
                                           digests=digests)
                for i, (allocation, offset) in enumerate(targets):
                    assert allocation.read_range(offset, size) == expected[i].tobytes(), f"{kind} block {i}"
                if save_mode == "staged":
                    label = f"{kind}/{chunk}"
                    if label in case["copies"]:
                        assert copies == case["copies"][label]
                    assert [list(d) for d in digests] == case["digests"]
                for allocation in owned:
                    allocation.close()
        # The KV cache was only read.
        after = host_bytes(tensors)
        assert all(np.array_equal(after[k], storages[k]) for k in storages)
    finally:
        plane.close()


@pytest.mark.parametrize("key", LARGE)
@pytest.mark.parametrize("restore_mode", ["direct", "staged"])
def test_load_scatter_restores_like_the_reference(key, restore_mode):
    case, storages, layout, tensors, caches = cuda_case(key)
    plane = plane_for(caches, restore_mode=restore_mode)
    try:
        packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        n, size = len(packed), plane.block_bytes
        owned, sources = targets_for(plane, "staging", n)
        for i, block in enumerate(packed):
            C.memmove(sources[i][0].pointer + sources[i][1], block.ctypes.data, size)
        progress = []
        launches = plane.load_scatter(case["restored"], sources, progress=progress,
                                      chunk_bytes=case["restore_chunk_bytes"])
        assert launches == case["launches"]
        assert [left for _, left in progress] == case["progress_left"]
        assert progress[0][0] is None and all(event.query() for event, _ in progress[1:])
        oracle.unpack(storages, layout, case["restored"], packed)
        after = host_bytes(tensors)
        assert {name: sha_of(buf) for name, buf in sorted(after.items())} == case["storage_sha256_after_restore"]
        assert all(np.array_equal(after[k], storages[k]) for k in storages)
        for allocation in owned:
            allocation.close()
    finally:
        plane.close()


@pytest.mark.parametrize("row", GOLDEN["small_layouts"], ids=lambda r: str(r["strides"]))
def test_small_stride_permutations_byte_for_byte(row):
    storages, tensors, caches = cuda_small(row)
    plane = plane_for(caches, block_size=4)
    try:
        owned, targets = targets_for(plane, "per-block", 2)
        digests = []
        plane.save_gather(row["saved"], targets, row["num_kv_tokens"], digests=digests)
        got = [a.read_range(0, plane.block_bytes).hex() for a, _ in targets]
        assert got == row["packed_hex"]
        assert [d[0] for d in digests] == [hashlib.sha256(bytes.fromhex(h)).hexdigest() for h in got]
        assert [d[1] for d in digests] == [oracle.crc32c(bytes.fromhex(h)) for h in got]
        plane.load_scatter(row["restored"], targets)
        assert host_bytes(tensors)["small"].tobytes().hex() == row["storage_hex_after_restore"]
    finally:
        plane.close()


def test_reference_gpu_round_trip_shape():
    """The reference's own GPU test geometry (tests/connector/test_copy_kernel_cuda.py:21-66):
    6 layers x 96 blocks, 20 shuffled blocks, three blocks a launch: seven launches, bit for bit."""
    layers, blocks = 6, 96
    raw = torch.from_numpy(kvgen.random_bytes(77, layers * blocks * 16 * 8 * 256 * 2)).cuda()
    backing = raw.view(torch.bfloat16).view(layers, blocks, 16, 8, 256)
    caches = {f"model.layers.{i}.self_attn.attn": backing[i].permute(0, 2, 1, 3) for i in range(layers)}
    plane = plane_for(caches)
    rng = random.Random(1)
    saved = rng.sample(range(1, blocks), 20)
    restored = rng.sample([b for b in range(1, blocks) if b not in saved], 20)
    size = plane.block_bytes
    try:
        before = backing.view(torch.int16).clone()
        for kind in ("staging", "per-block"):
            owned, targets = targets_for(plane, kind, len(saved))
            plane.save_gather(saved, targets, len(saved) * 16)
            progress = []
            assert plane.load_scatter(restored, targets, progress=progress, chunk_bytes=3 * size) == 7
            assert all(event.query() for event, _ in progress[1:])
            torch.cuda.synchronize()
            expected = before.clone()
            expected[:, restored] = before[:, saved]
            assert torch.equal(backing.view(torch.int16), expected)
            backing.view(torch.int16).copy_(before)
            for allocation in owned:
                allocation.close()
    finally:
        plane.close()


def test_verified_restore_rejects_a_corrupt_block_before_writing():
    case, storages, layout, tensors, caches = cuda_case("qwen3_8b_5d")
    plane = plane_for(caches)
    from kvsnap_b200.dataplane import CorruptBlockError
    try:
        packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        crcs = [oracle.crc32c(b) for b in packed]
        n, size = len(packed), plane.block_bytes
        owned, sources = targets_for(plane, "per-block", n)
        for (allocation, _), block in zip(sources, packed):
            C.memmove(allocation.pointer, block.ctypes.data, size)
        bad = 3
        flip = sources[bad][0].pointer + 12345
        C.memset(flip, C.string_at(flip, 1)[0] ^ 0x40, 1)
        before = host_bytes(tensors)
        progress = []
        with pytest.raises(CorruptBlockError) as err:
            plane.load_scatter(case["restored"], sources, progress=progress, expected_crc32c=crcs)
        assert err.value.blocks == [bad]
        assert progress == []                    # nothing reported: a miss
        after = host_bytes(tensors)
        assert all(np.array_equal(after[k], before[k]) for k in before)
        # Repaired, the same call restores and reports.
        C.memset(flip, C.string_at(flip, 1)[0] ^ 0x40, 1)
        assert plane.load_scatter(case["restored"], sources, progress=progress, expected_crc32c=crcs) == 1
        oracle.unpack(storages, layout, case["restored"], packed)
        after = host_bytes(tensors)
        assert all(np.array_equal(after[k], storages[k]) for k in storages)
    finally:
        plane.close()


def _dp():
    from kvsnap_b200.dataplane import _dp, _load
    return _dp(_load())


@pytest.mark.parametrize("hbm", [False, True])
@pytest.mark.parametrize("length", [8, 16, 24, 504, 512, 520, 4096 + 8, 65536, 65536 + 16, 3 * 65536 + 8, 1835008])
def test_crc32c_kernel_matches_the_reference_crc(length, hbm):
    lib = _dp()
    n = 5
    data = [kvgen.random_bytes(1000 + length + i, length) for i in range(n)]
    buf = torch.from_numpy(np.concatenate(data)).cuda()
    addrs = torch.tensor([buf.data_ptr() + i * length for i in range(n)], dtype=torch.int64, device="cuda")
    crc = torch.empty(n, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    vec = 16 if length % 16 == 0 else 8
    if hbm:
        vec |= 0x100          # KVSNAP_DP_HBM: the segment-lane kernel where the block allows it
    s = torch.cuda.current_stream().cuda_stream
    assert lib.kvsnap_dp_crc32c(addrs.data_ptr(), n, length, crc.data_ptr(), 0, status.data_ptr(), vec, 0, s) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert [v & 0xFFFFFFFF for v in crc.tolist()] == [oracle.crc32c(d.tobytes()) for d in data]


@pytest.mark.parametrize("length", [1, 8, 55, 56, 63, 64, 65, 119, 120, 128, 1000, 4096 + 48, 65536 + 8])
def test_sha256_kernel_matches_hashlib(length):
    lib = _dp()
    n = 33                       # two warps, the second with one lane
    data = [kvgen.random_bytes(5000 + length + i, length) for i in range(n)]
    stride = (length + 15) // 16 * 16
    host = np.zeros(n * stride, dtype=np.uint8)
    for i, d in enumerate(data):
        host[i * stride:i * stride + length] = d
    buf = torch.from_numpy(host).cuda()
    addrs = torch.tensor([buf.data_ptr() + i * stride for i in range(n)], dtype=torch.int64, device="cuda")
    out = torch.empty(n * 32, dtype=torch.uint8, device="cuda")
    assert lib.kvsnap_dp_sha256(addrs.data_ptr(), n, length, out.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    got = out.cpu().numpy().tobytes()
    assert [got[32 * i:32 * i + 32].hex() for i in range(n)] == [hashlib.sha256(d.tobytes()).hexdigest() for d in data]


def test_unaligned_sha256_source_takes_the_byte_path():
    lib = _dp()
    data = kvgen.random_bytes(4242, 1000)
    buf = torch.from_numpy(np.concatenate([np.zeros(3, np.uint8), data])).cuda()
    addrs = torch.tensor([buf.data_ptr() + 3], dtype=torch.int64, device="cuda")
    out = torch.empty(32, dtype=torch.uint8, device="cuda")
    assert lib.kvsnap_dp_sha256(addrs.data_ptr(), 1, 1000, out.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    assert out.cpu().numpy().tobytes().hex() == hashlib.sha256(data.tobytes()).hexdigest()


def test_pending_digests_arrive_after_the_save_returns():
    from kvsnap_b200.dataplane import PendingDigests
    case, storages, layout, tensors, caches = cuda_case("qwen3_1p7b_5d")
    plane = plane_for(caches)
    try:
        owned, targets = targets_for(plane, "per-block", len(case["saved"]))
        pending = PendingDigests()
        plane.save_gather(case["saved"], targets, case["num_kv_tokens"], digests=pending)
        expected = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        for i, (allocation, offset) in enumerate(targets):     # the bytes are there already
            assert allocation.read_range(offset, plane.block_bytes) == expected[i].tobytes()
        assert [list(d) for d in pending.result()] == case["digests"]
        assert pending.done() and pending.result() is pending.result()
        with pytest.raises(RuntimeError):
            PendingDigests().result()
    finally:
        plane.close()


def test_digest_of_pinned_blocks_matches_host_digest():
    case, storages, layout, tensors, caches = cuda_case("qwen3_1p7b_5d")
    plane = plane_for(caches)
    try:
        packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        owned, sources = targets_for(plane, "per-block", len(packed))
        for (allocation, _), block in zip(sources, packed):
            C.memmove(allocation.pointer, block.ctypes.data, plane.block_bytes)
        assert [list(d) for d in plane.digest(sources)] == case["digests"]
    finally:
        plane.close()


def test_copy_host_blocks_keeps_the_reference_kernel_interface():
    case, storages, layout, tensors, caches = cuda_case("vllm031")
    plane = plane_for(caches)
    from kvsnap_b200.dataplane import copy_host_blocks
    try:
        packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        owned, sources = targets_for(plane, "staging", len(packed))
        for i, block in enumerate(packed):
            C.memmove(sources[i][0].pointer + sources[i][1], block.ctypes.data, plane.block_bytes)
        tables = plane._load_tables()
        addresses = torch.tensor([a.pointer + o for a, o in sources], dtype=torch.int64, device="cuda")
        blocks = torch.tensor(case["restored"], dtype=torch.int64, device="cuda")
        copy_host_blocks(addresses, blocks, *tables)
        oracle.unpack(storages, layout, case["restored"], packed)
        after = host_bytes(tensors)
        assert np.array_equal(after["backing"], storages["backing"])
    finally:
        plane.close()


def test_ids_and_sources_are_checked_before_any_launch():
    case, storages, layout, tensors, caches = cuda_case("qwen3_8b_5d")
    plane = plane_for(caches)
    try:
        size = plane.block_bytes
        good = plane.pool.reserve(size)
        short = plane.pool.reserve(size - 16)
        closed = plane.pool.reserve(size)
        closed.close()
        before = host_bytes(tensors)
        for sources in ([(good, 0), (short, 0)], [(good, 0), (closed, 0)], [(good, -16), (good, 0)]):
            with pytest.raises((ValueError, RuntimeError)):
                plane.load_scatter([1, 2], sources)
        for ids in ([1, case["num_blocks"]], [1, -1], [1, 2.0]):
            with pytest.raises(ValueError):
                plane.load_scatter(ids, [(good, 0), (good, 0)])
        with pytest.raises(ValueError):
            plane.save_gather([1, 2], [(good, 0), (good, 0)], 33)   # 33 tokens need 3 blocks
        after = host_bytes(tensors)
        assert all(np.array_equal(after[k], before[k]) for k in before)
    finally:
        plane.close()
