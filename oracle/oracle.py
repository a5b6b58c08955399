"""ORACLE: a CPU restatement of kvsnap's KV snapshot data plane. Test infrastructure only.

Nothing in the product (``kvsnap_b200``) imports this module; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use it, and
only as the checker or the timed CPU reference, never as a code path that
serves results.

What it restates (reference paths are relative to the kvsnap source tree):

* Registration: layers packed in name order, each layer's block a dense span
  copied in storage order (``kvsnap/connector/dataplane.py:221-249``).
* Save: packed block i = concatenation, over the sorted layers, of that layer's
  span for ``block_ids[i]``; token slots at or past ``num_kv_tokens % block_size``
  of the last block are zeroed for every (layer, head) (``dataplane.py:262-272,
  388-437``; the gather itself is ``index_select`` + ``cat`` at 417).
* Restore: for each block and layer, the span at packed offset ``offset_l`` is
  written to ``base_l + block_ids[i] * pitch_l`` (``kvsnap/connector/copy_kernel.py:23-40``,
  ``dataplane.py:334-386``), one launch per ``chunk_bytes`` with progress
  ``[(None, total), (event, left)...]`` (``dataplane.py:356-379``).
* Save copy count: adjacent targets in one allocation share a copy, per chunk
  (``dataplane.py:406-427``).
* Checksums: CRC32C via the C restatement in ``oracle/crc32c.c`` (reference
  ``csrc/dataplane/io.cpp:16-47``); content id = ``hashlib.sha256(block).hexdigest()``
  (``kvsnap/store/store.py:616-629``, ``kvsnap/connector/volatile.py:141-151``).
* Dedup: one blob per distinct content id, segments keep every block
  (``store.py:625-628``, ``volatile.py:254-279``).
* Blob files: a 32-byte KVSBLOB1 header, then the packed block
  (``kvsnap/store/common.py:10-11``, ``blobs.py:33-36, 95-101``).
* TP regroup (no reference code exists; a TP-size mismatch is a miss there):
  defined by slicing the full-head KV by KV head, see ``slice_heads``.

Pinned by ``tests/test_oracle_golden.py`` against fixtures produced by running
the reference's own Python data plane and its compiled ``io.cpp`` (generator:
``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import hashlib
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = None


def _lib():
    """The C restatement (oracle/_build/liboracle.so), built by ``make -C oracle``."""
    global _LIB
    if _LIB is None:
        path = _HERE / "_build" / "liboracle.so"
        if not path.is_file():
            import subprocess
            subprocess.run(["make", "-s", "-C", str(_HERE), "_build/liboracle.so"], check=True)
        lib = ctypes.CDLL(str(path))
        for name in ("oracle_crc32c", "oracle_crc32c_bitwise"):
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32], ctypes.c_uint32
        lib.oracle_gf_mulmod.argtypes, lib.oracle_gf_mulmod.restype = [ctypes.c_uint32, ctypes.c_uint32], ctypes.c_uint32
        lib.oracle_xpow8n.argtypes, lib.oracle_xpow8n.restype = [ctypes.c_uint64], ctypes.c_uint32
        lib.oracle_crc32c_combine.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64]
        lib.oracle_crc32c_combine.restype = ctypes.c_uint32
        _LIB = lib
    return _LIB


def crc32c(data, prior: int = 0) -> int:
    """CRC32C of a bytes-like object (reference ``io.cpp:39-47``)."""
    buf = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
    return int(_lib().oracle_crc32c(buf.ctypes.data if buf.size else None, buf.size, prior))


def crc32c_bitwise(data, prior: int = 0) -> int:
    buf = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
    return int(_lib().oracle_crc32c_bitwise(buf.ctypes.data if buf.size else None, buf.size, prior))


def crc32c_combine(crc_a: int, crc_b: int, len_b: int) -> int:
    return int(_lib().oracle_crc32c_combine(crc_a, crc_b, len_b))


def gf_mulmod(a: int, b: int) -> int:
    return int(_lib().oracle_gf_mulmod(a, b))


def xpow8n(nbytes: int) -> int:
    return int(_lib().oracle_xpow8n(nbytes))


def sha256_hex(data) -> str:
    """The store's content id for one packed block (reference ``store.py:623``)."""
    return hashlib.sha256(memoryview(data).cast("B")).hexdigest()


# ---- layout ---------------------------------------------------------------

@dataclass
class Span:
    """One registered 4-D layer view, as the reference records it (``dataplane.py:245-247``).

    ``storage`` names a flat uint8 numpy buffer in the caller's ``storages``
    dict; ``start`` is the byte offset of block 0, ``pitch`` the byte stride
    between blocks, ``shape``/``stride`` the view's [H, N, C] dims and element
    strides, ``elem`` the element size in bytes.
    """
    name: str
    storage: str
    start: int
    pitch: int
    shape: tuple
    stride: tuple
    elem: int
    blocks: int
    offset: int = 0               # byte offset inside a packed block; set by ``register``

    @property
    def bytes(self) -> int:
        h, n, c = self.shape
        return h * n * c * self.elem


@dataclass
class Layout:
    spans: list
    block_size: int
    block_bytes: int = field(init=False)

    def __post_init__(self):
        offset = 0
        for span in self.spans:
            span.offset = offset
            offset += span.bytes
        self.block_bytes = offset


def register(views: dict, block_size: int) -> Layout:
    """Sort layers by name and check each is a dense [B,H,N,C] block (``dataplane.py:226-248``)."""
    if not views:
        raise ValueError("empty KV cache registration")
    spans = []
    for name in sorted(views):
        span = views[name]
        h, n, c = span.shape
        if n != block_size or span.stride[2] != 1:
            raise ValueError(f"unsupported KV layout for {name}")
        dense = 1
        for stride, size in sorted((s, d) for s, d in zip(span.stride, span.shape) if d > 1):
            if stride != dense:
                raise ValueError(f"unsupported KV layout for {name}: block has holes or overlapping axes")
            dense *= size
        if span.pitch // span.elem < dense:
            raise ValueError(f"unsupported KV layout for {name}: overlapping blocks")
        spans.append(span)
    return Layout(spans, block_size)


def split_5d(name: str, storage: str, start: int, num_blocks: int, block_size: int, heads: int,
             head_dim: int, elem: int) -> dict:
    """Two 4-D views of one ``[2, num_blocks, block_size, heads, head_dim]`` layer.

    ``name.k = t[0].permute(0, 2, 1, 3)`` and ``name.v = t[1].permute(0, 2, 1, 3)``:
    the registration that lets the reference's 4-D data plane take the 5-D
    paged layout, K before V within a layer.
    """
    half = num_blocks * block_size * heads * head_dim * elem
    pitch = block_size * heads * head_dim * elem
    shape = (heads, block_size, head_dim)
    stride = (head_dim, heads * head_dim, 1)
    return {f"{name}.{part}": Span(f"{name}.{part}", storage, start + i * half, pitch, shape, stride, elem,
                                   num_blocks)
            for i, part in enumerate(("k", "v"))}


def span_bytes(storages: dict, span: Span, block: int) -> np.ndarray:
    base = span.start + block * span.pitch
    return storages[span.storage][base:base + span.bytes]


# ---- save / restore -------------------------------------------------------

def zero_tail(layout: Layout, packed: np.ndarray, valid: int) -> None:
    """Zero token slots at or past ``valid`` in one packed block (``dataplane.py:262-272``)."""
    for span in layout.spans:
        h, n, c = span.shape
        sh, sn, _ = span.stride
        for head in range(h):
            for token in range(valid, n):
                at = span.offset + (head * sh + token * sn) * span.elem
                packed[at:at + c * span.elem] = 0


def pack(storages: dict, layout: Layout, block_ids, num_kv_tokens: int) -> list:
    """The packed snapshot blocks ``save_gather`` produces (``dataplane.py:388-437``)."""
    expected = (num_kv_tokens + layout.block_size - 1) // layout.block_size
    if len(block_ids) != expected:
        raise ValueError("block count does not cover computed tokens")
    blocks = []
    for block in block_ids:
        packed = np.empty(layout.block_bytes, dtype=np.uint8)
        for span in layout.spans:
            packed[span.offset:span.offset + span.bytes] = span_bytes(storages, span, block)
        blocks.append(packed)
    valid = num_kv_tokens % layout.block_size
    if valid and blocks:
        zero_tail(layout, blocks[-1], valid)
    return blocks


def unpack(storages: dict, layout: Layout, block_ids, packed_blocks) -> None:
    """Write packed blocks into ``block_ids`` in place (``copy_kernel.py:23-40``)."""
    if len(packed_blocks) != len(block_ids):
        raise ValueError("one source per block is required")
    for block, packed in zip(block_ids, packed_blocks):
        for span in layout.spans:
            base = span.start + block * span.pitch
            storages[span.storage][base:base + span.bytes] = packed[span.offset:span.offset + span.bytes]


def progress_lefts(n: int, block_bytes: int, chunk_bytes: int = 64 << 20) -> list:
    """Bytes left after each restore launch, led by the total (``dataplane.py:356-379``)."""
    per_launch = max(1, chunk_bytes // block_bytes)
    lefts = [n * block_bytes]
    for first in range(0, n, per_launch):
        lefts.append((n - min(n, first + per_launch)) * block_bytes)
    return lefts if n else []


def save_copy_count(targets, block_bytes: int, chunk_bytes: int = 64 << 20) -> int:
    """D2H copies ``save_gather`` issues: one per run of adjacent targets in one allocation, per chunk.

    ``targets[i]`` is ``(allocation_key, offset)`` (``dataplane.py:406-427``).
    """
    n = len(targets)
    if not n:
        return 0
    per_chunk = max(1, min(n, chunk_bytes // block_bytes))
    copies = 0
    for first in range(0, n, per_chunk):
        stop = min(n, first + per_chunk)
        i = first
        while i < stop:
            key, offset = targets[i]
            j = i + 1
            while j < stop and targets[j][0] == key and targets[j][1] == offset + (j - i) * block_bytes:
                j += 1
            copies += 1
            i = j
    return copies


def digests(blocks) -> list:
    """(content id, CRC32C) per packed block, as ``_prepare_payloads`` computes them."""
    return [(sha256_hex(b), crc32c(b)) for b in blocks]


def dedup(blocks) -> tuple:
    """Distinct blobs and per-block segments (``store.py:625-628``): returns (unique ids, segments)."""
    return dedup_digests(digests(blocks), [len(b) for b in blocks])


def dedup_digests(block_digests, lengths) -> tuple:
    """``dedup`` from per-block ``(content id, CRC32C)`` already computed: a payload dict keyed by
    content id keeps the first block of each (``store.py:625-628``, ``volatile.py:254-279``)."""
    unique, segments = {}, []
    for index, ((key, checksum), length) in enumerate(zip(block_digests, lengths)):
        unique.setdefault(key, index)
        segments.append(dict(blob_id=key, offset=0, length=length, first_block=index, nblocks=1, crc32c=checksum))
    return list(unique), segments


# ---- blob files ----------------------------------------------------------

# KVSBLOB1 header: magic, version 1, payload length, payload CRC32C, 8 reserved
# zero bytes, little-endian (kvsnap/store/common.py:10-11).
BLOB_HEADER = struct.Struct("<8sIQI8s")
BLOB_MAGIC = b"KVSBLOB1"


def blob_name(blob_id: str) -> str:
    """File name of a blob: its 64-hex content id plus ``.blob`` (``kvsnap/store/blobs.py:33-36``)."""
    if len(blob_id) != 64 or any(c not in "0123456789abcdef" for c in blob_id):
        raise ValueError("invalid blob identifier")
    return blob_id + ".blob"


def blob_file(payload) -> bytes:
    """The bytes of one blob file: header, then the payload (``kvsnap/store/blobs.py:95-101``)."""
    payload = bytes(payload)
    return BLOB_HEADER.pack(BLOB_MAGIC, 1, len(payload), crc32c(payload), bytes(8)) + payload


# ---- tensor-parallel shards -----------------------------------------------

def slice_heads(full: np.ndarray, tp: int, rank: int) -> np.ndarray:
    """Rank ``rank``'s KV-head shard of a full ``[2, B, N, H, D]`` layer at TP size ``tp``.

    The reference gives each TP rank heads ``[rank*H/tp, (rank+1)*H/tp)`` of its
    own KV cache and restores a snapshot only at the TP size it was saved at
    (``kvsnap/connector/vllm.py:9-14``). A TP-8 snapshot restored at TP-4 is
    therefore defined here as: TP-4 rank r must end up with exactly the heads a
    TP-4 save of the same KV would hold, i.e. this slice.
    """
    heads = full.shape[3]
    per = heads // tp
    return np.ascontiguousarray(full[:, :, :, rank * per:(rank + 1) * per, :])
