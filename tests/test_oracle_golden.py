"""Pin the CPU oracle to the reference: every golden vector the reference produced must come out of it.

The fixtures (tests/golden/golden.json) were made by running the reference's own
data plane, CRC32C library and hashlib (tests/golden/make_golden.py). A test
here failing means the oracle no longer restates the reference, so no parity
claim built on it holds.
"""
import numpy as np
import pytest

import kvgen
from cases import GOLDEN, golden_case, sha_of, storages_small
from oracle import oracle


def _data(row):
    return bytes.fromhex(row["hex"]) if "hex" in row else kvgen.random_bytes(row["seed"], row["length"]).tobytes()


@pytest.mark.parametrize("row", GOLDEN["crc32c"], ids=lambda r: r["label"])
def test_crc32c_matches_reference_vectors(row):
    data = _data(row)
    assert oracle.crc32c(data) == row["crc"]
    assert oracle.crc32c_bitwise(data) == row["crc"]
    if "crc_python_table" in row:
        assert row["crc_python_table"] == row["crc"]
    if "split" in row:
        s = row["split"]
        assert oracle.crc32c(data[s:], oracle.crc32c(data[:s])) == row["crc_extend"] == row["crc"]
        assert oracle.crc32c(data, 0x1234ABCD) == row["crc_prior_1234"]


def test_reference_known_answers():
    # The reference's own pins: tests/unit/test_native_io.py:99-103, tests/unit/test_store.py:41-44.
    assert oracle.crc32c(b"") == 0
    assert oracle.crc32c(b"123456789") == 0xE3069283
    assert oracle.crc32c(bytes(32)) == 0x8A9136AA
    assert oracle.crc32c(b"\xff" * 32) == 0x62A8AB43
    assert oracle.crc32c(b"456789", oracle.crc32c(b"123")) == 0xE3069283


def test_combine_rule_matches_direct_crc():
    data = kvgen.random_bytes(5, 10_000).tobytes()
    for split in (0, 1, 16, 4095, 9999, 10_000):
        a, b = data[:split], data[split:]
        assert oracle.crc32c_combine(oracle.crc32c(a), oracle.crc32c(b), len(b)) == oracle.crc32c(data)


@pytest.mark.parametrize("row", GOLDEN["registration"], ids=lambda r: str(r["strides"]))
def test_registration_accepts_and_rejects_like_the_reference(row):
    s = row["strides"]
    span = oracle.Span("layer.0", "x", 0, s[0] * 2, (3, 4, 8), tuple(s[1:]), 2, 5)
    if row["accepted"]:
        assert oracle.register({"layer.0": span}, 4).block_bytes == row["block_bytes"]
    else:
        with pytest.raises(ValueError):
            oracle.register({"layer.0": span}, 4)


@pytest.mark.parametrize("row", GOLDEN["small_layouts"], ids=lambda r: str(r["strides"]))
def test_small_layouts_pack_and_restore_byte_for_byte(row):
    storages, views = storages_small(row["strides"], row["seed"])
    layout = oracle.register(views, 4)
    packed = oracle.pack(storages, layout, row["saved"], row["num_kv_tokens"])
    assert [p.tobytes().hex() for p in packed] == row["packed_hex"]
    oracle.unpack(storages, layout, row["restored"], packed)
    assert storages["small"].tobytes().hex() == row["storage_hex_after_restore"]


@pytest.mark.parametrize("key", ["vllm031", "qwen3_1p7b_5d", "qwen3_8b_5d"])
def test_large_geometries_match_reference_digests_copies_and_progress(key):
    case, storages, layout = golden_case(key)
    assert layout.block_bytes == case["block_bytes"]
    assert [s.name for s in layout.spans] == [layer["name"] for layer in case["layers"]]
    packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
    assert [list(d) for d in oracle.digests(packed)] == case["digests"]
    size, n = layout.block_bytes, len(case["saved"])
    for label, copies in case["copies"].items():
        kind, chunk = label.split("/")
        targets = [(i, 0) for i in range(n)] if kind == "per-block" else [(0, i * size) for i in range(n)]
        assert oracle.save_copy_count(targets, size, int(chunk)) == copies, label
    assert oracle.progress_lefts(n, size, case["restore_chunk_bytes"]) == case["progress_left"]
    assert len(case["progress_left"]) - 1 == case["launches"]
    oracle.unpack(storages, layout, case["restored"], packed)
    assert {name: sha_of(buf) for name, buf in sorted(storages.items())} == case["storage_sha256_after_restore"]


def test_dedup_counts_identical_blocks_once():
    a = kvgen.random_bytes(1, 4096)
    b = kvgen.random_bytes(2, 4096)
    unique, segments = oracle.dedup([a, b, a.copy(), a])
    assert len(unique) == 2 and len(segments) == 4
    assert segments[2]["blob_id"] == segments[0]["blob_id"] == segments[3]["blob_id"]


def test_reshard_slice_is_the_tp4_shard_of_two_tp8_shards():
    full = kvgen.random_bytes(9, 2 * 3 * 16 * 8 * 128 * 2).view(np.uint16).reshape(2, 3, 16, 8, 128)
    for r in range(4):
        pair = np.concatenate([oracle.slice_heads(full, 8, 2 * r), oracle.slice_heads(full, 8, 2 * r + 1)], axis=3)
        assert np.array_equal(pair, oracle.slice_heads(full, 4, r))


def test_blob_files_equal_the_references():
    """The reference's BlobWriter wrote these files (tests/golden/make_golden.py, section 6)."""
    import hashlib
    g = GOLDEN["blobs"]
    payloads = [kvgen.random_bytes(seed, length).tobytes()
                for seed, length in zip(g["payload_seeds"], g["payload_lengths"])]
    blocks = [payloads[i] for i in g["blocks"]]
    assert oracle.dedup(blocks)[1] == g["segments"]
    for segment in g["segments"]:
        payload = blocks[segment["first_block"]]
        raw = oracle.blob_file(payload)
        want = g["files"][segment["blob_id"]]
        if "file_hex" in want:
            assert raw.hex() == want["file_hex"]
        else:
            assert raw[:32].hex() == want["header_hex"] and len(raw) == want["file_bytes"]
            assert hashlib.sha256(raw).hexdigest() == want["file_sha256"]
        assert oracle.blob_name(segment["blob_id"]) == segment["blob_id"] + ".blob"
