"""Blob files written from pinned memory (kvsnap_b200/blobs.py write_blobs), on the CPU.

The reference's BlobWriter wrote the golden files (tests/golden/make_golden.py,
section 6); write_blobs, given the same blocks and their (SHA-256, CRC32C)
digests, must leave byte-identical files and return the same segments. Plain
host buffers stand in for pinned allocations: write_blobs only reads them.
"""
import ctypes as C
import os

import pytest

import kvgen
from cases import GOLDEN
from oracle import oracle


class HostBlock:
    """What write_blobs reads of a pinned allocation: an open buffer's address and size."""

    def __init__(self, data: bytes):
        self.buffer = C.create_string_buffer(data, len(data))
        self.pointer, self.size = C.addressof(self.buffer), len(data)

    def _open(self):
        pass


def golden_blocks():
    g = GOLDEN["blobs"]
    payloads = [kvgen.random_bytes(seed, length).tobytes()
                for seed, length in zip(g["payload_seeds"], g["payload_lengths"])]
    return [payloads[i] for i in g["blocks"]]


@pytest.mark.parametrize("durability", ["process", "durable"])
def test_write_blobs_writes_the_references_files(tmp_path, durability):
    from kvsnap_b200.blobs import write_blobs
    g = GOLDEN["blobs"]
    blocks = golden_blocks()
    # One size per call, as packed blocks are: write the blocks of each size separately.
    for size in sorted({len(b) for b in blocks}):
        chosen = [i for i, b in enumerate(blocks) if len(b) == size]
        sources = [(HostBlock(blocks[i]), 0) for i in chosen]
        digests = [oracle.digests([blocks[i]])[0] for i in chosen]
        segments = write_blobs(tmp_path, sources, digests, size, durability=durability)
        want = [dict(s, first_block=k) for k, s in enumerate(g["segments"][i] for i in chosen)]
        assert segments == want
    files = sorted(os.listdir(tmp_path))
    assert files == sorted(oracle.blob_name(blob_id) for blob_id in g["files"])      # duplicates written once
    for blob_id, want in g["files"].items():
        raw = (tmp_path / oracle.blob_name(blob_id)).read_bytes()
        if "file_hex" in want:
            assert raw.hex() == want["file_hex"]
        else:
            assert raw[:32].hex() == want["header_hex"] and len(raw) == want["file_bytes"]


def test_existing_blobs_are_checked_not_rewritten(tmp_path):
    from kvsnap_b200.blobs import write_blobs
    from kvsnap_b200.dataplane import CorruptBlockError
    data = kvgen.random_bytes(5, 4096).tobytes()
    digest = oracle.digests([data])[0]
    write_blobs(tmp_path, [(HostBlock(data), 0)], [digest], 4096, durability="process")
    path = tmp_path / oracle.blob_name(digest[0])
    before = path.stat().st_mtime_ns
    write_blobs(tmp_path, [(HostBlock(data), 0)], [digest], 4096, durability="durable")
    assert path.stat().st_mtime_ns == before and path.read_bytes() == oracle.blob_file(data)
    # A file under that name whose header no longer describes the block is refused, as in the reference.
    raw = bytearray(path.read_bytes())
    raw[20] ^= 1                                         # the header's CRC32C field
    path.write_bytes(bytes(raw))
    with pytest.raises(CorruptBlockError, match="differs"):
        write_blobs(tmp_path, [(HostBlock(data), 0)], [digest], 4096)
    assert sorted(os.listdir(tmp_path)) == [path.name]  # no temporary file left behind


def test_write_blobs_rejects_bad_arguments(tmp_path):
    from kvsnap_b200.blobs import write_blobs
    from kvsnap_b200.dataplane import CorruptBlockError
    data = bytes(64)
    digest = oracle.digests([data])[0]
    with pytest.raises(CorruptBlockError, match="identifier"):
        write_blobs(tmp_path, [(HostBlock(data), 0)], [("XYZ", 0)], 64)
    with pytest.raises(ValueError, match="outside"):
        write_blobs(tmp_path, [(HostBlock(data), 16)], [digest], 64)
    with pytest.raises(ValueError, match="durability"):
        write_blobs(tmp_path, [(HostBlock(data), 0)], [digest], 64, durability="volatile")
    with pytest.raises(ValueError, match="one digest"):
        write_blobs(tmp_path, [(HostBlock(data), 0)], [], 64)
    assert write_blobs(tmp_path, [], [], 64) == [] and os.listdir(tmp_path) == []
