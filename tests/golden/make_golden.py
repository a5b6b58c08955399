"""Generate tests/golden/golden.json by running the REFERENCE kvsnap data plane on the CPU.

    python tests/golden/make_golden.py --reference <kvsnap source tree>

Needs the reference source tree (read-only) and ``make -C oracle REF=<tree>``
(which compiles the reference's own ``csrc/dataplane/io.cpp`` into
``oracle/_ref/libkvsnap_io_ref.so``). Everything recorded here is produced by
the reference's code, never by this repository's product:

* ``TorchBlockDataPlane`` (reference ``kvsnap/connector/dataplane.py``) is
  registered on CPU tensors with CUDA calls replaced by no-ops, the pinned pool
  by host buffers whose copies are memmoves, and the restore kernel by a
  memmove per (block, layer) job over the tables the data plane builds (the
  Triton kernel's semantics, ``kvsnap/connector/copy_kernel.py:23-40``);
* CRC32C comes from ``kvsnap.store.crc32c.crc32c`` bound to the compiled
  reference ``io.cpp`` (and, for short inputs, its pure-Python table path);
* content ids are ``hashlib.sha256(block).hexdigest()`` as in
  ``kvsnap/store/store.py:623``.

Inputs are regenerated from seeds by ``tests/kvgen.py``, so the fixture stores
seeds, block tables and results, not cache contents.
"""
from __future__ import annotations

import argparse
import contextlib
import ctypes as C
import hashlib
import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace
from unittest.mock import patch

import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO / "tests"))
import kvgen  # noqa: E402

sys.path.insert(0, str(REPO))
from oracle.refharness import HostBuffer, register, restore_by_memmove  # noqa: E402


# ---- the CUDA-free stand-ins live in oracle/refharness.py ---------------------

# ---- cache geometries -------------------------------------------------------

def caches_5d(seed, layers, num_blocks, block_size, heads, head_dim, prefix="model.layers"):
    """Per layer one ``[2, num_blocks, block_size, heads, head_dim]`` bf16 tensor (the paged layout),
    registered as two 4-D views ``name.k``/``name.v`` (``t[i].permute(0, 2, 1, 3)``)."""
    caches, backings = {}, {}
    per_layer = 2 * num_blocks * block_size * heads * head_dim * 2
    for i in range(layers):
        raw = torch.from_numpy(kvgen.random_bytes(seed * 1000 + i, per_layer))
        tensor = raw.view(torch.bfloat16).view(2, num_blocks, block_size, heads, head_dim)
        backings[f"{prefix}.{i}"] = tensor
        caches[f"{prefix}.{i}.k"] = tensor[0].permute(0, 2, 1, 3)
        caches[f"{prefix}.{i}.v"] = tensor[1].permute(0, 2, 1, 3)
    return caches, backings


def caches_vllm031(seed, layers, num_blocks, block_size=16, heads=8, width=256):
    """vLLM 0.31.0's registration: per layer a [B, H, N, C] view of [B, N, H, C] storage,
    K and V side by side in C, all layers carved from one buffer."""
    nbytes = layers * num_blocks * block_size * heads * width * 2
    raw = torch.from_numpy(kvgen.random_bytes(seed, nbytes))
    backing = raw.view(torch.bfloat16).view(layers, num_blocks, block_size, heads, width)
    return {f"model.layers.{i}.self_attn.attn": backing[i].permute(0, 2, 1, 3) for i in range(layers)}, backing


def storage_sha(tensor):
    t = tensor.contiguous()
    return hashlib.sha256(C.string_at(t.data_ptr(), t.numel() * t.element_size())).hexdigest()


def save_case(dataplane, crc32c, caches, block_size, saved, restored, tokens, chunk_blocks, backing_tensors):
    plane = register(dataplane, caches, block_size)
    size = plane.block_bytes
    out = {"block_bytes": size, "layers": plane.layers, "saved": saved, "restored": restored,
           "num_kv_tokens": tokens}
    # Per-block targets (host tier) and one staging buffer (disk), default and small chunks.
    for kind in ("per-block", "staging"):
        for chunk in (64 << 20, chunk_blocks * size):
            if kind == "per-block":
                targets = [(HostBuffer(size), 0) for _ in saved]
            else:
                staged = HostBuffer(size * len(saved))
                targets = [(staged, i * size) for i in range(len(saved))]
            copies = plane.save_gather(saved, targets, tokens, chunk_bytes=chunk)
            out.setdefault("copies", {})[f"{kind}/{chunk}"] = copies
            blocks = [a.read_range(o, size) for a, o in targets]
            digests = [[hashlib.sha256(b).hexdigest(), crc32c(b)] for b in blocks]
            out.setdefault("digests", digests)
            assert out["digests"] == digests, "packed blocks depend on the target kind"
    # Restore the staged snapshot into other blocks, chunked, and record what moved.
    staged = HostBuffer(size * len(saved))
    targets = [(staged, i * size) for i in range(len(saved))]
    plane.save_gather(saved, targets, tokens)
    progress = []
    with patch.object(dataplane, "copy_host_blocks", new=restore_by_memmove):
        launches = plane.load_scatter(restored, targets, progress=progress, chunk_bytes=chunk_blocks * size)
    out["launches"] = launches
    out["restore_chunk_bytes"] = chunk_blocks * size
    out["progress_left"] = [left for _, left in progress]
    out["storage_sha256_after_restore"] = {name: storage_sha(t) for name, t in sorted(backing_tensors.items())}
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="the kvsnap source tree (read-only)")
    parser.add_argument("--out", default=str(Path(__file__).resolve().parent / "golden.json"))
    args = parser.parse_args()
    ref_io = REPO / "oracle/_ref/libkvsnap_io_ref.so"
    if not ref_io.is_file():
        raise SystemExit("build the reference io library first: make -C oracle")
    os.environ["KVSNAP_IO_LIBRARY"] = str(ref_io)
    sys.path.insert(0, args.reference)
    from kvsnap.connector import dataplane
    from kvsnap.store.crc32c import crc32c
    crc_module = sys.modules["kvsnap.store.crc32c"]
    from kvsnap.store.native_io import PythonIO, get_io_backend
    assert get_io_backend().name == "native"

    golden = {"generator": "tests/golden/make_golden.py", "reference_io": "csrc/dataplane/io.cpp"}

    # 1. CRC32C: the reference's known vectors, and lengths / splits / priors through its native library,
    #    with its pure-Python table path alongside for the short ones.
    vectors = []
    python_io = PythonIO()
    for label, data in [("empty", b""), ("123456789", b"123456789"), ("zeros32", bytes(32)),
                        ("ones32", b"\xff" * 32), ("range256x4", bytes(range(256)) * 4)]:
        vectors.append({"label": label, "hex": data.hex(), "crc": crc32c(data)})
    for seed, length in [(1, 1), (2, 7), (3, 15), (4, 16), (5, 17), (6, 63), (7, 64), (8, 65), (9, 4095),
                         (10, 4096), (11, 65536 + 24)]:
        data = kvgen.random_bytes(seed, length).tobytes()
        row = {"label": f"random/{seed}/{length}", "seed": seed, "length": length, "crc": crc32c(data)}
        if length <= 4096:
            with patch.object(crc_module, "get_io_backend", return_value=SimpleNamespace(name="python")):
                row["crc_python_table"] = crc32c(data)
        split = length // 3
        row["split"] = split
        row["crc_extend"] = crc32c(data[split:], crc32c(data[:split]))
        row["crc_prior_1234"] = crc32c(data, 0x1234ABCD)
        vectors.append(row)
    golden["crc32c"] = vectors

    # 2. Registration: accepted and rejected stride sets (reference layout tests' geometry).
    layouts = []
    for strides in [(96, 8, 24, 1), (192, 32, 8, 1), (96, 32, 8, 1), (192, 8, 24, 1), (96, 8, 8, 1),
                    (48, 32, 8, 1)]:
        storage = torch.zeros(5 * max(strides[0], 96) + 256, dtype=torch.bfloat16)
        cache = storage.as_strided((5, 3, 4, 8), strides)
        try:
            plane = register(dataplane, {"layer.0": cache}, 4)
            layouts.append({"strides": list(strides), "accepted": True, "block_bytes": plane.block_bytes,
                            "layers": plane.layers})
        except ValueError as exc:
            layouts.append({"strides": list(strides), "accepted": False, "error": str(exc)})
    golden["registration"] = layouts

    # 3. Small stride permutations: full packed bytes, tail zeroing, restore.
    small = []
    for strides in [(96, 32, 8, 1), (96, 8, 24, 1), (192, 32, 8, 1), (192, 8, 24, 1)]:
        raw = torch.from_numpy(kvgen.random_bytes(strides[0] + strides[1], 5 * strides[0] * 2))
        storage = raw.view(torch.bfloat16)
        cache = storage.as_strided((5, 3, 4, 8), strides)
        plane = register(dataplane, {"layer.0": cache}, 4)
        targets = [(HostBuffer(plane.block_bytes), 0) for _ in range(2)]
        plane.save_gather([1, 3], targets, 6)
        packed = [a.read_range(0, plane.block_bytes).hex() for a, _ in targets]
        with patch.object(dataplane, "copy_host_blocks", new=restore_by_memmove):
            plane.load_scatter([0, 4], targets)
        small.append({"strides": list(strides), "seed": strides[0] + strides[1], "saved": [1, 3],
                      "num_kv_tokens": 6, "packed_hex": packed, "restored": [0, 4],
                      "storage_hex_after_restore": C.string_at(storage.data_ptr(), storage.numel() * 2).hex()})
    golden["small_layouts"] = small

    # 4. vLLM 0.31.0 4-D geometry (36 layers, 64 KiB spans), 12-block cache.
    caches, backing = caches_vllm031(seed=31, layers=36, num_blocks=12)
    case = save_case(dataplane, crc32c, caches, 16, [7, 2, 9, 3, 4], [10, 0, 5, 6, 1], 4 * 16 + 5, 2,
                     {"backing": backing})
    case.update({"kind": "vllm031", "seed": 31, "layers": case["layers"], "num_layers": 36, "num_blocks": 12})
    golden["vllm031"] = case

    # 5. The paged 5-D layout through the two-view registration, Qwen3-1.7B and Qwen3-8B shaped.
    for key, seed, layers, num_blocks, saved_n, tokens in [("qwen3_1p7b_5d", 17, 28, 24, 8, 7 * 16 + 9),
                                                           ("qwen3_8b_5d", 8, 36, 20, 6, 6 * 16)]:
        caches, backings = caches_5d(seed, layers, num_blocks, 16, 8, 128)
        saved, restored = kvgen.disjoint_block_sets(seed, num_blocks, saved_n)
        case = save_case(dataplane, crc32c, caches, 16, saved, restored, tokens, 3, backings)
        case.update({"kind": "5d", "seed": seed, "num_layers": layers, "num_blocks": num_blocks,
                     "heads": 8, "head_dim": 128})
        golden[key] = case

    # 6. Blob files: the reference's BlobWriter.prepare_blocks (kvsnap/store/store.py:647-674) on
    #    seeded payloads, one of them twice (dedup). Recorded: the segments it returns and each
    #    KVSBLOB1 file it wrote (whole file for short payloads, header + SHA-256 for long ones).
    import tempfile
    from kvsnap.store.store import BlobWriter
    payloads = [kvgen.random_bytes(60 + i, length).tobytes()
                for i, length in enumerate([16, 4096, 65536 + 48])]
    blocks = [payloads[0], payloads[1], payloads[0], payloads[2]]
    with tempfile.TemporaryDirectory() as root:
        record = BlobWriter(root).prepare_blocks(blocks, durability="process")
        files = {}
        for segment in record["segments"]:
            raw = (Path(root) / "blobs" / (segment["blob_id"] + ".blob")).read_bytes()
            files[segment["blob_id"]] = ({"file_hex": raw.hex()} if len(raw) <= 8192 else
                                         {"header_hex": raw[:32].hex(), "file_sha256": hashlib.sha256(raw).hexdigest(),
                                          "file_bytes": len(raw)})
    golden["blobs"] = {"payload_seeds": [60, 61, 62], "payload_lengths": [16, 4096, 65536 + 48],
                       "blocks": [0, 1, 0, 2], "segments": record["segments"], "files": files}

    Path(args.out).write_text(json.dumps(golden, indent=1, sort_keys=True) + "\n")
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
