"""Snapshot blobs between pinned memory and disk, with the GPU's checksums.

The reference's disk tier hashes on the host on both sides.

Save (``BlobWriter.prepare_blocks``, ``kvsnap/store/store.py:647-674``):
- copies every packed block into a Python ``bytes`` object;
- hashes it with SHA-256 and CRC32C on eight host threads (``_prepare_payloads``, ``store.py:616-629``);
- writes each distinct content id as a KVSBLOB1 file (``blobs.py:78-111``).

Restore (``BlobWriter.read_prepared_into``, ``store.py:676-713``):
- reads every block into pinned staging;
- CRCs it on the host;
- only then does the connector start any host-to-device copy (``vllm.py:495-499``).

This module keeps the file format and the failure rules and moves the arithmetic to the GPU:

* :func:`write_blobs` writes each block straight from its pinned allocation: one pwrite from the
  pinned address, no bytes object. The file is named by the SHA-256 content id and headed by the
  CRC32C that ``save_gather(..., digests=)`` computed on the GPU, and a content id seen twice is
  written once.
* :func:`read_and_restore` has reader threads pread blocks into pinned staging. Meanwhile, as each
  chunk of consecutive blocks lands, the GPU copies it into device staging and checks its CRC32Cs
  against the manifest, so disk reads, host-to-device copies and checks overlap. The KV cache is
  written only after every block has passed, so a corrupt or unreadable blob leaves it untouched
  and reports no progress, as the reference's restore does.
"""
from __future__ import annotations

import fcntl
import os
import struct
import uuid
from concurrent.futures import ThreadPoolExecutor
from contextlib import contextmanager
from pathlib import Path

from . import _abi
from .dataplane import CorruptBlockError, _dp, _u32

# KVSBLOB1 header: magic, version, payload length, payload CRC32C, 8 reserved
# zero bytes, little-endian (reference kvsnap/store/common.py:10-11).
HEADER = struct.Struct("<8sIQI8s")
MAGIC = b"KVSBLOB1"
VERSION = 1
_HEX = set("0123456789abcdef")


def blob_path(blob_dir, blob_id) -> Path:
    """``<blob_dir>/<content id>.blob`` (reference blobs.py:33-36)."""
    if not isinstance(blob_id, str) or len(blob_id) != 64 or not set(blob_id) <= _HEX:
        raise CorruptBlockError("invalid blob identifier")
    return Path(blob_dir) / (blob_id + ".blob")


_pools = {}


def _io(io, workers):
    """The caller's I/O backend, or a native pread/pwrite pool of ``workers`` threads for this process."""
    if io is not None:
        return io
    from .native_io import NativeIO, resolve_io_library
    key = (os.getpid(), max(2, workers))
    if key not in _pools:
        _pools[key] = NativeIO(resolve_io_library(), workers=key[1], queue_bytes=256 << 20)
    return _pools[key]


@contextmanager
def _shared_lock(lock_path):
    """The store's ``.blob.lock``, shared, when the caller names one (reference store.py:703-705)."""
    if lock_path is None:
        yield
        return
    with open(lock_path, "a+b") as lock_file:
        fcntl.flock(lock_file, fcntl.LOCK_SH)
        yield


def _sync_directory(path):
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _check_existing(path, length, checksum):
    """A blob already under this content id: its header must describe this payload (reference blobs.py:62-77)."""
    try:
        with open(path, "rb") as stream:
            raw = stream.read(HEADER.size)
            size = os.fstat(stream.fileno()).st_size
    except OSError as exc:
        raise CorruptBlockError(f"existing blob {path.name} is unreadable: {exc}") from exc
    if len(raw) != HEADER.size:
        raise CorruptBlockError("truncated blob header")
    magic, version, size_field, crc_field, reserved = HEADER.unpack(raw)
    if (magic != MAGIC or version != VERSION or reserved != bytes(8) or size_field != size - HEADER.size
            or size_field != length or crc_field != checksum):
        raise CorruptBlockError(f"existing blob {path.name} differs from the block it names")


def write_blobs(blob_dir, sources, digests, block_bytes, *, durability="durable", io=None, workers=8):
    """Write packed blocks from pinned memory as KVSBLOB1 files named by their content ids.

    ``sources[i]`` is ``(allocation, offset)`` holding packed block i of
    ``block_bytes`` bytes (for example the targets ``save_gather`` wrote),
    ``digests[i]`` its ``(sha256 hex, crc32c)`` from
    ``save_gather(..., digests=)``. A content id
    that appears twice, or whose file already exists with a matching header, is
    written once. Each new blob goes to a temporary file (header, then the
    payload straight from pinned memory), is fdatasynced when ``durability`` is
    "durable", and is renamed into place; the directory is fsynced once at the
    end (reference blobs.py:78-111, store.py:665-674). Returns the segments the
    store's manifest records: ``{blob_id, offset 0, length, first_block i,
    nblocks 1, crc32c}`` per block (store.py:625-628).
    """
    if durability not in ("process", "durable"):
        raise ValueError("blob durability is process or durable")
    if len(sources) != len(digests):
        raise ValueError("one digest per block is required")
    if type(block_bytes) is not int or block_bytes <= 0:
        raise ValueError("block_bytes must be a positive integer")
    io = _io(io, workers)
    blob_dir = Path(blob_dir)
    size = block_bytes
    segments, unique = [], {}
    for index, ((allocation, offset), (blob_id, checksum)) in enumerate(zip(sources, digests)):
        allocation._open()
        if offset < 0 or offset + size > allocation.size:
            raise ValueError("blob source outside its allocation")
        path = blob_path(blob_dir, blob_id)
        segments.append(dict(blob_id=blob_id, offset=0, length=size, first_block=index, nblocks=1,
                             crc32c=int(checksum)))
        unique.setdefault(blob_id, (path, allocation, offset, int(checksum)))

    def write(item):
        path, allocation, offset, checksum = item
        if path.exists():
            _check_existing(path, size, checksum)
            if durability == "durable":
                fd = os.open(path, os.O_RDONLY)
                try:
                    os.fdatasync(fd)
                finally:
                    os.close(fd)
            return
        temporary = path.with_name(path.name[:-5] + "." + uuid.uuid4().hex + ".tmp")
        fd = os.open(temporary, os.O_CREAT | os.O_EXCL | os.O_WRONLY, 0o600)
        try:
            io.pwrite_all(fd, HEADER.pack(MAGIC, VERSION, size, checksum, bytes(8)), 0)
            allocation._open()
            io.pwrite_from(fd, allocation.pointer + offset, size, HEADER.size)
            if durability == "durable":
                os.fdatasync(fd)
        except BaseException:
            os.close(fd)
            os.unlink(temporary)
            raise
        os.close(fd)
        os.replace(temporary, path)

    if unique:
        with ThreadPoolExecutor(max_workers=max(1, workers), thread_name_prefix="kvsnap-blob-write") as pool:
            list(pool.map(write, unique.values()))
        if durability == "durable":
            _sync_directory(blob_dir)
    return segments


def _read_block(io, blob_dir, segment, address, size):
    """One blob's header check and one pread of its payload into ``address`` (reference store.py:689-700)."""
    blob_id = segment["blob_id"]
    try:
        fd = os.open(blob_path(blob_dir, blob_id), os.O_RDONLY)
        try:
            raw = io.pread_all(fd, HEADER.size, 0)
            if len(raw) != HEADER.size:
                raise CorruptBlockError("truncated blob header")
            magic, version, length, _, reserved = HEADER.unpack(raw)
            if magic != MAGIC or version != VERSION or reserved != bytes(8) or segment["offset"] + size > length:
                raise CorruptBlockError("invalid blob header or segment bounds")
            io.pread_into(fd, address, size, HEADER.size + segment["offset"])
        finally:
            os.close(fd)
    except (OSError, struct.error) as exc:
        raise CorruptBlockError(f"unreadable blob {blob_id}: {exc}") from exc


def read_and_restore(plane, blob_dir, segments, block_ids, staged, *, first_block=0, io=None, workers=8,
                     chunk_bytes=64 << 20, progress=None, lock_path=None, cache=None, generations=None):
    """Restore a disk-tier snapshot: blob reads, host-to-device copies and GPU CRC checks overlapped.

    ``segments``: the manifest's segments of the blocks restored here, block
    ``first_block + i`` into cache block ``block_ids[i]`` (reference
    store.py:676-688 checks them the same way). ``staged``: a pinned
    allocation of at least ``len(block_ids) * plane.block_bytes`` bytes that
    receives the packed blocks in order. ``lock_path``: the store's
    ``.blob.lock``, held shared while reading, as the reference does.

    Reader threads pread blocks in order; as soon as a chunk of consecutive
    blocks has landed, the restore's copy stream moves it into device staging
    and its CRC32Cs are checked there against the manifest. Once every block
    has passed, the scatter kernel writes them into the KV cache, one launch per
    ``chunk_bytes``, and ``progress`` receives ``(None, total)`` and then
    ``(event, bytes left)`` per launch, as ``load_scatter`` reports them. An
    unreadable blob, a bad header or a checksum mismatch raises
    :class:`CorruptBlockError` (its ``blocks`` lists the mismatching block
    indices) before any KV byte is written. Returns the scatter launch count.

    ``cache`` (a ``DigestCache``) and ``generations``: once restored, each
    block with a generation is recorded under it with its segment's content
    id and CRC32C, so the next save of an unchanged block skips SHA-256.
    """
    torch = plane.torch
    plane._validate_ids(block_ids)
    n, size = len(block_ids), plane.block_bytes
    if len(segments) != n:
        raise ValueError("one segment per block is required")
    if (cache is None) != (generations is None) or (generations is not None and len(generations) != n):
        raise ValueError("a digest cache needs one generation per block")
    for index, segment in enumerate(segments, start=first_block):
        if segment["first_block"] != index or segment["nblocks"] != 1:
            raise CorruptBlockError("noncontiguous prepared block mapping")
        offset, length = segment["offset"], segment["length"]
        if type(offset) is not int or type(length) is not int or offset < 0 or length != size:
            raise CorruptBlockError("prepared segment does not match the KV block size")
    if n == 0:
        return 0
    if staged.size < n * size:
        raise ValueError("staging allocation is smaller than the blocks it receives")
    staged.wait()                       # no earlier copy may still read the bytes the reads overwrite
    io = _io(io, workers)
    lib = _dp(plane.pool.lib)
    spans = plane._spans()
    plane._scatter_targets()
    device = plane._device()
    copies, kernels = plane._load_copy_stream, plane._load_stream
    per_chunk = max(1, chunk_bytes // size)
    vec = (16 | plane._hbm) if size % 16 == 0 else 8
    expected = [segment["crc32c"] for segment in segments]
    with torch.cuda.stream(kernels):
        stage = torch.empty(n * size, dtype=torch.uint8, device=device)
        stage.record_stream(copies)
        table = torch.tensor([stage.data_ptr() + i * size for i in range(n)], dtype=torch.int64).pin_memory().to(
            device, non_blocking=True)
        ids = torch.tensor(list(block_ids), dtype=torch.int64).pin_memory().to(device, non_blocking=True)
        expect = torch.tensor(_u32(expected), dtype=torch.int32).pin_memory().to(device, non_blocking=True)
        crc = torch.empty(n, dtype=torch.int32, device=device)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        allocated = torch.cuda.Event()
        allocated.record(kernels)
    copies.wait_event(allocated)

    # 1. Reads land chunk by chunk; each landed chunk is copied and checked on the GPU.
    reads = ThreadPoolExecutor(max_workers=max(1, workers), thread_name_prefix="kvsnap-blob-read")
    futures = []
    try:
        with _shared_lock(lock_path):
            futures = [reads.submit(_read_block, io, blob_dir, segments[i], staged.pointer + i * size, size)
                       for i in range(n)]
            for first in range(0, n, per_chunk):
                last = min(n, first + per_chunk)
                for future in futures[first:last]:
                    future.result()
                plane.pool.copy_many([(staged, first * size, stage.data_ptr() + first * size, (last - first) * size)],
                                     to_host=False, stream=copies.cuda_stream)
                landed = torch.cuda.Event()
                landed.record(copies)
                kernels.wait_event(landed)
                plane._check(lib.kvsnap_dp_crc32c(table[first:].data_ptr(), last - first, size, crc[first:].data_ptr(),
                                                  expect[first:].data_ptr(), status.data_ptr(), vec, plane.ctas,
                                                  kernels.cuda_stream))
    except BaseException:
        for future in futures:
            future.cancel()
        reads.shutdown(wait=True)
        copies.synchronize()
        kernels.synchronize()
        raise
    reads.shutdown(wait=True)
    kernels.synchronize()
    flags = int(status.item())
    if flags & _abi.CRC_MISMATCH:
        got = [v & 0xFFFFFFFF for v in crc.tolist()]
        bad = [i for i, (g, e) in enumerate(zip(got, expected)) if g != e]
        raise CorruptBlockError(f"prepared segment checksum mismatch at block index {bad[0]}", bad)
    if flags:
        plane._status_error(status)

    # 2. Every block passed: scatter from device staging into the cache.
    if progress is not None:
        progress.append((None, n * size))
    launches, done = 0, None
    with torch.cuda.stream(kernels):
        for first in range(0, n, per_chunk):
            last = min(n, first + per_chunk)
            plane._check(lib.kvsnap_dp_scatter(spans.data_ptr(), len(plane.layers), size, table[first:].data_ptr(),
                                               ids[first:].data_ptr(), last - first, 0, 0, 0, status.data_ptr(), vec,
                                               plane.ctas, kernels.cuda_stream))
            launches += 1
            done = torch.cuda.Event()
            done.record(kernels)
            if progress is not None:
                progress.append((done, (n - last) * size))
    done.synchronize()
    plane._status_error(status)
    if cache is not None:
        for block, generation, segment in zip(block_ids, generations, segments):
            if generation is not None:
                cache.put(block, generation, (segment["blob_id"], segment["crc32c"]))
    return launches
