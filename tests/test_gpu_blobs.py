"""The disk tier on a B200: save -> KVSBLOB1 files -> verified restore, against the oracle.

save_gather's GPU digests name and head the blob files write_blobs writes from
pinned memory; read_and_restore reads them back into pinned staging while the
GPU copies and CRC-checks each landed chunk, then scatters into other cache
blocks. The restored cache must equal the oracle's unpack of the oracle's
packed blocks. A flipped payload byte, a damaged header or a missing file must
raise CorruptBlockError before any KV byte is written and with no progress
reported (the reference's restore turns the same cases into a miss).
"""
import numpy as np
import pytest
import torch

from cases import golden_case
from gpu_cases import cuda_5d, host_bytes
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def disk_case(tmp_path):
    from kvsnap_b200.blobs import write_blobs
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    case, storages, layout = golden_case("qwen3_8b_5d")
    _, tensors, caches = cuda_5d(case)
    plane = TorchBlockDataPlane(caches, 16, 256 << 20)
    # A block repeated away from the (tail-zeroed) last slot: one blob, two segments.
    saved = list(case["saved"][:3]) + [case["saved"][0]] + list(case["saved"][3:])
    tokens = len(saved) * 16 - 5                             # a partial last block
    size = plane.block_bytes
    snapshot = plane.pool.reserve(len(saved) * size)
    targets = [(snapshot, i * size) for i in range(len(saved))]
    digests = []
    plane.save_gather(saved, targets, tokens, digests=digests)
    segments = write_blobs(tmp_path, targets, digests, size, durability="durable")
    packed = oracle.pack(storages, layout, saved, tokens)
    yield plane, tmp_path, segments, packed, storages, layout, tensors, saved
    plane.close()


def test_blob_round_trip_restores_like_the_oracle(disk_case):
    from kvsnap_b200.blobs import read_and_restore
    plane, blob_dir, segments, packed, storages, layout, tensors, saved = disk_case
    assert [s["crc32c"] for s in segments] == [oracle.crc32c(b) for b in packed]
    assert len({s["blob_id"] for s in segments}) == len(saved) - 1
    restored = [10, 11, 12, 13, 14, 15, 16][: len(saved)]
    size = plane.block_bytes
    for chunk in (64 << 20, 2 * size):                      # one chunk, then chunks of two blocks
        staged = plane.pool.reserve(len(saved) * size)
        progress = []
        launches = read_and_restore(plane, blob_dir, segments, restored, staged, chunk_bytes=chunk,
                                    progress=progress)
        expected_launches = -(-len(saved) // max(1, chunk // size))
        assert launches == expected_launches
        assert progress[0] == (None, len(saved) * size) and progress[-1][1] == 0
        assert all(event.query() for event, _ in progress[1:])
        staged.close()
    oracle.unpack(storages, layout, restored, packed)
    after = host_bytes(tensors)
    assert all(np.array_equal(after[k], storages[k]) for k in storages)


@pytest.mark.parametrize("damage", ["payload", "header", "missing"])
def test_damaged_blobs_raise_before_any_kv_write(disk_case, damage):
    from kvsnap_b200.blobs import blob_path, read_and_restore
    from kvsnap_b200.dataplane import CorruptBlockError
    plane, blob_dir, segments, packed, storages, layout, tensors, saved = disk_case
    victim = 2
    path = blob_path(blob_dir, segments[victim]["blob_id"])
    if damage == "payload":
        raw = bytearray(path.read_bytes())
        raw[32 + 12345] ^= 0x40
        path.write_bytes(bytes(raw))
    elif damage == "header":
        raw = bytearray(path.read_bytes())
        raw[0] ^= 1                                          # the magic
        path.write_bytes(bytes(raw))
    else:
        path.unlink()
    before = host_bytes(tensors)
    staged = plane.pool.reserve(len(saved) * plane.block_bytes)
    progress = []
    with pytest.raises(CorruptBlockError) as raised:
        read_and_restore(plane, blob_dir, segments, [10, 11, 12, 13, 14, 15, 16][: len(saved)], staged,
                         chunk_bytes=2 * plane.block_bytes, progress=progress)
    if damage == "payload":
        assert raised.value.blocks == [victim]
    assert progress == []
    after = host_bytes(tensors)
    assert all(np.array_equal(after[k], before[k]) for k in before)
    staged.close()


def test_segments_are_checked_first(disk_case):
    from kvsnap_b200.blobs import read_and_restore
    from kvsnap_b200.dataplane import CorruptBlockError
    plane, blob_dir, segments, packed, storages, layout, tensors, saved = disk_case
    staged = plane.pool.reserve(len(saved) * plane.block_bytes)
    with pytest.raises(CorruptBlockError, match="noncontiguous"):
        read_and_restore(plane, blob_dir, segments, list(range(10, 10 + len(saved))), staged, first_block=1)
    short = [dict(s, length=s["length"] - 16) for s in segments]
    with pytest.raises(CorruptBlockError, match="block size"):
        read_and_restore(plane, blob_dir, short, list(range(10, 10 + len(saved))), staged)
    with pytest.raises(ValueError, match="one segment"):
        read_and_restore(plane, blob_dir, segments[:-1], list(range(10, 10 + len(saved))), staged)
    staged.close()
