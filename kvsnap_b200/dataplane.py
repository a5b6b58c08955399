"""The KV snapshot data plane: a drop-in for kvsnap's ``kvsnap.connector.dataplane``.

Same module surface as the reference (kvsnap/connector/dataplane.py):
``resolve_cuda_library``, ``copy_host_blocks``, ``PinnedCapacityError``,
``CudaPool``, ``PinnedAllocation`` and ``TorchBlockDataPlane`` with the
constructor, attributes (``caches``, ``block_size``, ``layers``,
``block_bytes``, ``pool``) and methods the connector uses (``warm_up``,
``staging``, ``producer_event``, ``wait_on_engine_stream``, ``load_scatter``,
``save_gather``, ``close``), the same argument meaning, return values and
exceptions. The copies run in sm_100a kernels from ``_cuda_native.so``
(include/kvsnap_cuda.h) instead of torch ops and a Triton kernel, and the
checksums the store needs are computed on the GPU in the same call:

* ``save_gather(..., digests=out)`` fills ``out`` with ``(sha256 hex, crc32c)``
  per block, the values kvsnap/store/store.py:616-629 and
  kvsnap/connector/volatile.py:141-151 compute on the host;
* ``load_scatter(..., expected_crc32c=crcs)`` checks every block's CRC32C on
  the GPU before any KV byte is written (the check kvsnap/store/store.py:717-718
  runs on the loader thread), raising :class:`CorruptBlockError` on a mismatch.

There is no CPU path: without the CUDA library or a CUDA device these raise.
"""
from __future__ import annotations

import collections
import ctypes as C
import os
import threading
from contextlib import contextmanager
from importlib.machinery import EXTENSION_SUFFIXES
from pathlib import Path

from . import _abi

_NATIVE = Path(__file__).resolve().parent / "_native"


def resolve_cuda_library(library=None):
    """The C ABI library's path, without loading it or initialising CUDA (reference dataplane.py:12-25).

    ``library`` or ``KVSNAP_CUDA_LIBRARY`` wins; otherwise this package's
    ``_native/_cuda_native<suffix>`` built by ``python -m kvsnap_b200.build``.
    """
    override = library or os.environ.get("KVSNAP_CUDA_LIBRARY")
    if override:
        return Path(override)
    for suffix in EXTENSION_SUFFIXES:
        candidate = _NATIVE / ("_cuda_native" + suffix)
        if candidate.is_file():
            return candidate
    packaged = sorted(_NATIVE.glob("_cuda_native*.so"))
    return packaged[0] if packaged else _NATIVE / "_cuda_native.so"


def _load(library=None):
    path = resolve_cuda_library(library)
    if not path.is_file():
        raise RuntimeError(f"kvsnap CUDA library not found at {path}; build it with python -m kvsnap_b200.build")
    lib = _abi.load(path, _abi.POOL_API)
    _abi.declare(lib, _abi.POOL_EXTRA, required=False)
    _abi.declare(lib, _abi.DP_API, required=False)
    return lib


def _dp(lib):
    """The library's data-plane entry points, or an error naming what is missing."""
    if not hasattr(lib, "kvsnap_dp_abi_version") or lib.kvsnap_dp_abi_version.restype is None:
        raise RuntimeError("the CUDA library has no data-plane kernels; rebuild with python -m kvsnap_b200.build")
    if lib.kvsnap_dp_abi_version() != _abi.DP_ABI_VERSION:
        raise RuntimeError("unsupported kvsnap data-plane ABI; rebuild with python -m kvsnap_b200.build")
    return lib


def copy_host_blocks(sources, blocks, layer_offsets, layer_bases, layer_pitches, layer_words):
    """The reference restore kernel's launch (copy_kernel.py:43-49), on the current stream.

    ``sources``: address of each packed block (pinned host or device memory);
    ``blocks``: its target block id; the ``layer_*`` tables: per layer, its
    offset in a packed block, the cache's base address and block pitch in bytes,
    and its span in 8-byte words. All int64 CUDA tensors.
    """
    import torch
    lib = _dp(_load())
    tables = (sources, blocks, layer_offsets, layer_bases, layer_pitches, layer_words)
    for table in tables:
        if table.dtype != torch.int64 or not table.is_cuda or not table.is_contiguous():
            raise ValueError("copy_host_blocks takes contiguous int64 CUDA tensors")
    if sources.numel() != blocks.numel():
        raise ValueError("one source per block is required")
    stream = torch.cuda.current_stream(sources.device).cuda_stream
    rc = lib.kvsnap_dp_copy_host_blocks(sources.data_ptr(), blocks.data_ptr(), sources.numel(),
                                        layer_offsets.data_ptr(), layer_bases.data_ptr(), layer_pitches.data_ptr(),
                                        layer_words.data_ptr(), layer_offsets.numel(), 0, stream)
    if rc < 0:
        raise RuntimeError(lib.kvsnap_cuda_error().decode())


class PinnedCapacityError(MemoryError):
    """The pinned pool cannot fit a reservation. Nothing was copied."""


class CorruptBlockError(ValueError):
    """A packed block's CRC32C differs from the one recorded for it. No KV byte was written."""

    def __init__(self, message, blocks=()):
        super().__init__(message)
        self.blocks = list(blocks)


class PendingDigests:
    """Content ids and CRC32Cs of a save whose SHA-256 kernel may still be running.

    Pass one as ``save_gather(..., digests=PendingDigests())``: the call returns
    once the packed blocks are in pinned memory, and ``result()`` later waits for
    the digest kernel and returns ``[(sha256 hex, crc32c), ...]`` in block order.
    """

    def __init__(self):
        self._event = None
        self._finish = None
        self._value = None

    def _bind(self, event, finish):
        # `finish` holds the staging buffer until the kernel reading it is done,
        # and turns the kernels' outputs into the list once `event` has passed.
        self._event, self._finish = event, finish

    def done(self) -> bool:
        return self._value is not None or (self._event is not None and self._event.query())

    def result(self):
        if self._value is None:
            if self._event is None:
                raise RuntimeError("no save has been bound to these digests")
            self._event.synchronize()
            self._value = self._finish()
            self._finish = None
        return self._value


class DigestCache:
    """Known content ids of GPU KV blocks, so that a save hashes only the blocks a turn changed.

    An entry maps (GPU block id, generation) to the ``(sha256 hex, crc32c)`` of
    that block's packed bytes. The generation is the caller's: it must change
    whenever the engine writes the block or the block is allocated anew (a
    full vLLM block is immutable until it is freed). ``save_gather`` and
    ``load_scatter`` fill the cache for the full blocks they move; a save then
    skips SHA-256 for every full block it finds, after checking that the CRC32C
    it just computed on the GPU equals the cached one (a mismatch is hashed
    after all and counted in ``rejected``). The reference hashes every block of
    every save (kvsnap/store/store.py:616-629, connector/volatile.py:141-151)
    and lists "hashing only the blocks a turn changed" as its next step.
    Least recently used entries go first beyond ``capacity``.

    What the cache trusts: the generation is the guarantee that a block's bytes
    are unchanged; the CRC32C comparison only catches a caller that broke that
    contract. A block that changed without a new generation and whose new bytes
    happen to have the same CRC32C (one chance in 2**32 a block) would be given
    the old content id, and a content-addressed store would file it under
    another block's bytes. Callers that cannot keep the generation contract
    should not pass a cache: then every block is hashed.
    """

    def __init__(self, capacity: int = 1 << 20):
        if type(capacity) is not int or capacity <= 0:
            raise ValueError("digest cache capacity must be a positive integer")
        self.capacity = capacity
        self._entries = collections.OrderedDict()
        self._lock = threading.Lock()
        self.hits = self.misses = self.rejected = 0

    def get(self, block, generation):
        with self._lock:
            entry = self._entries.get((block, generation))
            if entry is not None:
                self._entries.move_to_end((block, generation))
            return entry

    def put(self, block, generation, digest):
        sha, crc = digest
        if not isinstance(sha, str) or len(sha) != 64:
            raise ValueError("a digest is (64-hex sha256, crc32c)")
        with self._lock:
            self._entries[(block, generation)] = (sha, int(crc) & 0xFFFFFFFF)
            self._entries.move_to_end((block, generation))
            while len(self._entries) > self.capacity:
                self._entries.popitem(last=False)

    def forget(self, blocks):
        """Drop every generation of these blocks (for example when the engine frees them)."""
        blocks = set(blocks)
        with self._lock:
            for key in [k for k in self._entries if k[0] in blocks]:
                del self._entries[key]

    def __len__(self):
        return len(self._entries)


def _nonnegative(*values):
    if min(values) < 0:
        raise ValueError("negative copy argument")


class CudaPool:
    """A pinned host arena and its copy stream, owned through the C ABI v2 (reference dataplane.py:38-131).

    Every entry point refuses a pool inherited across fork or already closed,
    and runs under the pool's re-entrant lock, so a close waits for an
    operation in progress. The Python allocation objects are kept until the
    native pool has drained, because the native side may still be copying for
    them; a close that cannot drain the copy stream raises and leaves the
    pool, its allocations and their tensor owners intact.
    """

    def __init__(self, capacity_bytes: int, device: int = 0, library=None, *, shared_name=None):
        self._pid = os.getpid()
        self._lock = threading.RLock()
        self._allocations = {}
        self.lib = _load(library)
        self.abi_version = self.lib.kvsnap_pool_abi_version()
        if self.abi_version != _abi.POOL_ABI_VERSION:
            raise RuntimeError("unsupported kvsnap CUDA pool ABI; rebuild both CUDA and torch extensions")
        self.device = device
        # A shared pool's arena is POSIX shared memory other processes of this user map by name
        # (kvsnap_b200.sharedtier), so they read its blocks in place instead of over a socket.
        self.shared_name = shared_name
        if shared_name is None:
            self.handle = self.lib.kvsnap_pool_create(capacity_bytes, device)
        else:
            if not hasattr(self.lib, "kvsnap_pool_create_shared"):
                raise RuntimeError("this CUDA library has no shared pools; rebuild with python -m kvsnap_b200.build")
            self.handle = self.lib.kvsnap_pool_create_shared(capacity_bytes, device, shared_name.encode())
        if not self.handle:
            raise RuntimeError(self._error())

    def _error(self):
        return self.lib.kvsnap_cuda_error().decode()

    def _not_forked(self):
        if self._pid != os.getpid():
            raise RuntimeError("CUDA pools must not be inherited across fork")

    def _native(self, entry, *args):
        """Pool entry point ``entry`` on this pool's handle; a negative result raises with the library's message."""
        result = getattr(self.lib, entry)(self.handle, *args)
        if result < 0:
            raise RuntimeError(self._error())
        return result

    def check(self, result):
        if result < 0:
            raise RuntimeError(self._error())
        return result

    @contextmanager
    def operation(self):
        self._not_forked()
        with self._lock:
            if not self.handle:
                raise RuntimeError("pool closed")
            yield

    def reserve(self, size):
        ident, pointer = C.c_uint64(), C.c_void_p()
        with self.operation():
            if self.lib.kvsnap_pool_reserve(self.handle, size, C.byref(ident), C.byref(pointer)) < 0:
                message = self._error()
                full = "pinned capacity exhausted" in message
                raise PinnedCapacityError(message) if full else RuntimeError(message)
            allocation = PinnedAllocation(self, ident.value, pointer.value, size)
            self._allocations[allocation.ident] = allocation
        return allocation

    def close(self):
        self._not_forked()
        with self._lock:
            if not self.handle:
                return
            self._native("kvsnap_pool_close_checked")     # raises, keeping everything, when the drain fails
            self.handle = None
            for allocation in self._allocations.values():
                allocation._retire()
            self._allocations = {}

    def copy_many(self, entries, *, to_host, stream=0):
        """Queue copies ``(allocation, offset, device_ptr, size)`` in order on ``stream`` in one native call.

        ``stream`` 0 is the pool's copy stream; another stream orders its own
        producers. Every entry is checked before any copy is queued; each
        allocation's completion event covers all of them (kvsnap_pool_copy_many).
        """
        with self.operation():
            if not entries:
                return
            for allocation, offset, device_ptr, size in entries:
                self._owns(allocation)
                _nonnegative(offset, device_ptr, size, stream)
            columns = zip(*((a.ident, offset, ptr, size) for a, offset, ptr, size in entries))
            arrays = [(C.c_uint64 * len(entries))(*column) for column in columns]
            self._native("kvsnap_pool_copy_many", len(entries), *arrays, int(bool(to_host)), stream)

    def wait_many(self, allocations):
        """``wait`` for each allocation, in one native call (kvsnap_pool_wait_many)."""
        with self.operation():
            allocations = list(allocations)
            for allocation in allocations:
                self._owns(allocation)
            if allocations:
                ids = (C.c_uint64 * len(allocations))(*(a.ident for a in allocations))
                self._native("kvsnap_pool_wait_many", len(allocations), ids)

    def arena(self):
        """``(address of the arena's first byte, capacity)``: an allocation lies at ``pointer - address``."""
        with self.operation():
            base, capacity = C.c_void_p(), C.c_size_t()
            self._native("kvsnap_pool_arena", C.byref(base), C.byref(capacity))
            return base.value, capacity.value

    def _owns(self, allocation):
        if allocation.pool is not self:
            raise ValueError("allocation belongs to another pool")
        allocation._open()

    def stream_handle(self) -> int:
        """The copy stream's handle (borrowed; valid while the pool is open)."""
        with self.borrow_copy_stream() as handle:
            return handle

    @contextmanager
    def borrow_copy_stream(self):
        """Borrow the copy stream's handle; the context excludes a concurrent close (reference dataplane.py:110-131)."""
        with self.operation():
            handle = C.c_size_t()
            self._native("kvsnap_pool_copy_stream", C.byref(handle))
            if not handle.value:
                raise RuntimeError("native copy stream handle is invalid")
            yield handle.value


class PinnedAllocation:
    """One reservation in a :class:`CudaPool`: pinned bytes and the id its copies are fenced under
    (reference dataplane.py:134-211).

    Callers may hang the tensors a copy still reads on ``_tensor_references``;
    they are let go once the allocation is waited for or retired.
    """

    def __init__(self, pool, ident, pointer, size):
        self.pool, self.ident, self.pointer, self.size = pool, ident, pointer, size
        self.closed = False

    def _open(self):
        if self.closed or not self.pool.handle:
            raise RuntimeError("pinned allocation closed")

    def _drop_owners(self):
        owners = getattr(self, "_tensor_references", None)
        if owners is not None:
            owners.clear()

    def _retire(self):
        self.closed = True
        self._drop_owners()

    @contextmanager
    def operation(self):
        with self.pool.operation():
            self._open()
            yield

    def _native(self, entry, *args):
        return self.pool._native(entry, self.ident, *args)

    def copy(self, device_ptr, size, offset=0, *, to_host, producer_stream=0):
        with self.operation():
            _nonnegative(size, offset, device_ptr, producer_stream)
            self._native("kvsnap_pool_copy", offset, device_ptr, size, int(bool(to_host)), producer_stream)

    def copy_2d(self, device_ptr, device_pitch, host_offset, host_pitch, width, height, *,
                to_host, producer_stream=0):
        """``height`` rows of ``width`` bytes between strided device and host memory."""
        with self.operation():
            _nonnegative(device_ptr, device_pitch, host_offset, host_pitch, width, height, producer_stream)
            self._native("kvsnap_pool_copy_2d", host_offset, host_pitch, device_ptr, device_pitch, width, height,
                         int(bool(to_host)), producer_stream)

    def copy_on(self, device_ptr, size, offset=0, *, to_host, stream):
        """Like :meth:`copy`, queued on ``stream`` instead of the pool's copy stream (no producer fence)."""
        with self.operation():
            _nonnegative(size, offset, device_ptr, stream)
            self._native("kvsnap_pool_copy_on", offset, device_ptr, size, int(bool(to_host)), stream)

    def mark(self, stream=0):
        """Fence work queued so far on ``stream`` (0: the pool's copy stream) under this allocation's
        wait/ready/release: kernels that read or write the allocation in place run there, and
        marking after them makes the allocation's lifetime cover them."""
        with self.operation():
            self._native("kvsnap_pool_mark", stream)

    def wait(self):
        with self.operation():
            self._native("kvsnap_pool_wait")
            self._drop_owners()

    def ready(self):
        with self.operation():
            return bool(self._native("kvsnap_pool_ready"))

    def _settled(self, offset, size, what):
        """Wait for the allocation's copies; then the address of bytes [offset, offset + size) of it."""
        self.wait()
        if type(offset) is not int or type(size) is not int or offset < 0 or size < 0 or offset + size > self.size:
            raise ValueError(f"pinned {what} outside allocation")
        return self.pointer + offset

    def read(self):
        with self.operation():
            return C.string_at(self._settled(0, self.size, "read"), self.size)

    def read_range(self, offset, size):
        with self.operation():
            return C.string_at(self._settled(offset, size, "read"), size)

    def zero(self, offset, size):
        with self.operation():
            C.memset(self._settled(offset, size, "zero"), 0, size)

    def write(self, data):
        with self.operation():
            self.wait()
            if len(data) != self.size:
                raise ValueError("pinned allocation length mismatch")
            C.memmove(self.pointer, data, self.size)

    def close(self):
        pool = self.pool
        pool._not_forked()
        with pool._lock:
            if not self.closed and pool.handle:
                self._native("kvsnap_pool_release")
            pool._allocations.pop(self.ident, None)
            self._retire()


def _split_paged(caches, block_size):
    """Registered 4-D views: a 5-D ``[2, B, block_size, H, D]`` layer becomes ``name.k`` / ``name.v``.

    Both are ``t[i].permute(0, 2, 1, 3)``, a [B, H, N, D] view of [B, N, H, D]
    storage, K before V in name order: the registration under which the
    reference's 4-D data plane packs a paged FlashAttention cache.
    """
    views = {}
    for name, tensor in caches.items():
        shape = tuple(getattr(tensor, "shape", ()))
        if getattr(tensor, "ndim", 0) == 5 and shape[0] == 2 and shape[2] == block_size:
            views[f"{name}.k"] = tensor[0].permute(0, 2, 1, 3)
            views[f"{name}.v"] = tensor[1].permute(0, 2, 1, 3)
        else:
            views[name] = tensor
    return views


def _layer_record(name, tensor, block_size, device):
    """The reference's record of one registered layer view, after its checks (reference dataplane.py:230-247).

    Every view lives on the one CUDA ``device``. A view is ``[blocks, heads, tokens, width]`` with ``block_size`` tokens and
    contiguous width. Its per-block axes may be permuted in storage (vLLM's
    ``[blocks, tokens, heads, width]`` seen as BHNC) but must tile one dense
    span: taken in order of stride, each axis longer than 1 has the stride
    of the product of the smaller ones. Blocks may be further apart than a
    span, never closer. The record keeps the actual shape, dtype and strides.
    """
    if tensor.device != device or tensor.device.type != "cuda":
        raise ValueError("one CUDA device required")
    shape, strides = tuple(tensor.shape), tuple(tensor.stride()) if tensor.ndim else ()
    if tensor.ndim != 4 or shape[2] != block_size or strides[3] != 1:
        raise ValueError(f"unsupported KV layout for {name}: need dense [B,H,N,C] blocks with contiguous C")
    span = 1
    for stride, size in sorted((strides[axis], shape[axis]) for axis in (1, 2, 3) if shape[axis] > 1):
        if stride != span:
            raise ValueError(f"unsupported KV layout for {name}: block has holes or overlapping axes")
        span *= size
    if strides[0] < span:
        raise ValueError(f"unsupported KV layout for {name}: overlapping blocks")
    return {"name": name, "shape": list(shape[1:]), "dtype": str(tensor.dtype), "stride": list(strides[1:]),
            "bytes": shape[1] * shape[2] * shape[3] * tensor.element_size()}


def _even_pitch(targets, first, end, size):
    """The pitch at which targets[first:end] lie, if one pitch (at least ``size``) spaces them all, else None."""
    if end - first == 1:
        return size
    pitch = targets[first + 1] - targets[first]
    if pitch < size:
        return None
    for i in range(first + 2, end):
        if targets[i] - targets[i - 1] != pitch:
            return None
    return pitch


def column_plan(span_bytes, n, slot_bytes):
    """How a staged save moves through device slots of ``slot_bytes`` when its blocks do not fit at once.

    Every block of a group is moved a column at a time: a column is a run of
    consecutive spans, the same for every block, so a slot holds that column
    of ``group`` blocks, each ``stride`` bytes apart. Columns end at a multiple
    of 64 bytes into the block (SHA-256 goes in 64-byte chunks), except the
    last, and are about ``slot_bytes / n`` bytes, at least one span. Returns
    ``(group, stride, columns)``, each column ``(first span, end span, byte
    offset in the block, bytes)``; ``group * stride <= slot_bytes`` unless one
    column of one block is larger than a slot.
    """
    if n <= 0 or not span_bytes:
        raise ValueError("a column plan needs blocks and spans")
    target = max(64, slot_bytes // n // 64 * 64)
    columns, first, offset, size = [], 0, 0, 0
    for s, nbytes in enumerate(span_bytes):
        if size and size + nbytes > target and offset % 64 == 0:
            columns.append((first, s, offset - size, size))
            first, size = s, 0
        size += nbytes
        offset += nbytes
    columns.append((first, len(span_bytes), offset - size, size))
    stride = (max(c[3] for c in columns) + 15) // 16 * 16
    group = max(1, min(n, slot_bytes // stride))
    return group, stride, columns


def _u32(values):
    """Python ints in [0, 2**32) as the int32 bit patterns a torch int32 tensor holds."""
    return [v - (1 << 32) if v >= 1 << 31 else v for v in values]


class _SaveJob:
    """One save's state: what it moves, and the device buffers its digests still read."""

    def __init__(self, block_ids, targets, valid, hashed, known, digests):
        self.block_ids, self.targets, self.valid = block_ids, targets, valid
        self.hashed, self.known, self.digests = hashed, known, digests
        self.status = self.crc = self.digest = self.side = self.keep = None
        self.land = None                 # the stream its columns land on by the copy engine, if any
        self.rehash_from = []


class TorchBlockDataPlane:
    """Packed physical blocks: layer-name order, dense [H,N,C] stride permutations (reference dataplane.py:214-249).

    The actual layout is recorded and compared; unsupported views fail closed.
    Allocations stay live until the copies that touch them complete, including
    on error paths.

    ``save_mode``: ``"staged"`` gathers into device memory and moves the packed
    blocks to pinned memory with the copy engine (the default, and always
    used when digests are requested); ``"direct"`` has the gather kernel
    write the pinned blocks in place over the host link. ``restore_mode``:
    ``"staged"`` moves pinned blocks to a device ring with the copy engine and
    scatters them from there (the default: copy engines in both directions at
    once reach about twice what one direction does, SM reads of host memory
    beside a copy do not); ``"direct"`` has the scatter kernel read pinned
    blocks in place. A restore with ``expected_crc32c`` checks every block
    before any KV byte changes.

    ``staging_bytes`` bounds the device memory one call stages through (512
    MiB by default; the engine's KV cache owns the rest of the GPU): a save
    whose packed blocks exceed it moves through a ring of ``staging_slots``
    device slots a column of spans at a time; a verified restore that exceeds
    it checks the CRCs over the pinned blocks first and then restores through
    the two-slot chunk ring; ``digest`` hashes the pinned blocks in place. A
    restore's chunk ring holds two ``chunk_bytes`` chunks.

    ``column_landing``: how such a save's columns reach pinned memory.
    ``"kernel"`` (the default): a landing kernel stores them through the SMs.
    ``"copy"``: where a group's targets lie at one pitch (blocks reserved back
    to back, or one buffer), one copy-engine transfer a column on a stream of
    its own, overlapping the gather of the next column; other targets still
    land by kernel. On B200 a lone 8k Qwen3-8B save took 22.5 ms with "copy"
    against 24.8 with "kernel", but with restores running at the same time
    (a serving worker's connector threads) "copy" moved 5 % fewer bytes a
    second end to end, so it suits saves that run alone.

    ``shared_name`` puts the pinned pool in POSIX shared memory of that name, so
    that other workers restore its host-tier blocks in place
    (:mod:`kvsnap_b200.sharedtier`).
    """

    save_mode = "staged"
    restore_mode = "staged"
    staging_slots = 8
    sha_sms = 16

    def __init__(self, caches, block_size, capacity_bytes, *, save_mode=None, restore_mode=None, ctas=0,
                 staging_bytes=512 << 20, shared_name=None, column_landing="kernel"):
        import torch
        if not caches:
            raise ValueError("empty KV cache registration")
        self.torch = torch
        self.caches = dict(sorted(_split_paged(caches, block_size).items()))
        self.block_size = block_size
        device = next(iter(self.caches.values())).device
        self.layers = [_layer_record(name, tensor, block_size, device) for name, tensor in self.caches.items()]
        self.block_bytes = sum(layer["bytes"] for layer in self.layers)
        self.save_mode = save_mode or self.save_mode
        self.restore_mode = restore_mode or self.restore_mode
        if self.save_mode not in ("staged", "direct") or self.restore_mode not in ("staged", "direct"):
            raise ValueError("save_mode and restore_mode are 'staged' or 'direct'")
        self.ctas = ctas
        if type(staging_bytes) is not int or staging_bytes < (1 << 20):
            raise ValueError("staging_bytes must be an int of at least 1 MiB")
        self.staging_bytes = staging_bytes
        if column_landing not in ("kernel", "copy"):
            raise ValueError("column_landing is 'kernel' or 'copy'")
        self.column_landing = column_landing
        # Kernels that read or write pinned memory in place are bound by the host
        # link, which 16-32 CTAs already saturate; the rest of the GPU stays free
        # for the engine and the SHA-256 kernel.
        self.host_ctas = ctas or 32
        self.pool = CudaPool(capacity_bytes, device.index, shared_name=shared_name)

    @property
    def hbm_ctas(self):
        """CTAs of a device-memory gather, scatter or CRC launch.

        Those kernels' CTAs each take most of an SM's shared memory, so one
        cannot start on an SM where a SHA-256 CTA (of this save or another
        session's) runs: launched on every SM, a gather or scatter would wait
        for that hash, tens of milliseconds, to finish. Unless ``ctas`` was
        given, they leave ``sha_sms`` SMs to the hashes.
        """
        return self._grid_beside(0)

    def _grid_beside(self, hashed_blocks):
        """``hbm_ctas``, leaving at least the SMs a hash of ``hashed_blocks`` blocks occupies (64 blocks an SM)."""
        if self.ctas:
            return self.ctas
        if getattr(self, "_sm_count", None) is None:
            self._sm_count = self.torch.cuda.get_device_properties(self._device()).multi_processor_count
        return max(1, self._sm_count - max(self.sha_sms, (hashed_blocks + 63) // 64))

    # ---- registration-time tables ------------------------------------------------------------

    def _device(self):
        return next(iter(self.caches.values())).device

    def _spans(self):
        """The device span table (include/kvsnap_cuda.h ``kvsnap_span``), built on first use."""
        if getattr(self, "_span_table", None) is None:
            torch = self.torch
            lib = _dp(self.pool.lib)
            spans = (_abi.Span * len(self.layers))()
            vec = 16
            for span, layer, tensor in zip(spans, self.layers, self.caches.values()):
                size = tensor.element_size()
                base, pitch = tensor.data_ptr(), tensor.stride(0) * size
                if pitch % 8 or base % 8 or layer["bytes"] % 8:
                    raise ValueError(f"KV layer {layer['name']} is not 8-byte aligned for the scatter path")
                if pitch % 16 or base % 16 or layer["bytes"] % 16:
                    vec = 8
                span.base, span.pitch, span.bytes = base, pitch, layer["bytes"]
                span.token_pitch = tensor.stride(2) * size
                span.tokens, span.row_bytes = tensor.shape[2], tensor.shape[3] * size
                span.nblocks = tensor.shape[0]
            total = C.c_uint64()
            if lib.kvsnap_dp_plan(spans, len(spans), C.byref(total)) < 0:
                raise RuntimeError(lib.kvsnap_cuda_error().decode())
            if total.value != self.block_bytes:
                raise RuntimeError("packed block size disagrees with the registered layers")
            host = torch.frombuffer(bytearray(bytes(spans)), dtype=torch.uint8)
            self._span_vec = vec
            # Device-side copies may use the segment-lane HBM kernels, with the unit cut that the
            # layer sizes allow.
            self._hbm = _abi.hbm_flags([layer["bytes"] for layer in self.layers], vec)
            self._min_blocks = min(t.shape[0] for t in self.caches.values())
            self._span_table = host.to(self._device())
            # Side streams: restores that read pinned memory in place run on their
            # own stream, so one can overlap a save's copies (the host link is full
            # duplex); digests run on streams of their own, so concurrent saves'
            # SHA-256 kernels overlap each other and the copies.
            self._load_stream = torch.cuda.Stream(self._device())
            self._load_copy_stream = torch.cuda.Stream(self._device())
            self._sha_streams = [torch.cuda.Stream(self._device()) for _ in range(4)]
            # A bounded save's columns land by the copy engine on a stream of their own, so the
            # gather of the next column overlaps the landing of this one.
            self._land_stream = torch.cuda.Stream(self._device())
            self._sha_next = 0
            self._sha_lock = threading.Lock()
        return self._span_table

    def _scatter_targets(self):
        """Build the tables on first use and borrow the pool's copy stream as a torch stream."""
        self._spans()
        if getattr(self, "_copy_stream", None) is None:
            with self.pool.borrow_copy_stream() as handle:
                self._copy_stream = self.torch.cuda.ExternalStream(handle, device=self._device())
        return self._copy_stream

    def _load_tables(self):
        """Per layer, as int64 device tensors: its offset in a packed block, its cache's base address and
        block pitch in bytes, and its span in 8-byte words (the tables of :func:`copy_host_blocks`)."""
        if getattr(self, "_tables", None) is None:
            self._scatter_targets()
            columns, offset = ([], [], [], []), 0
            for layer, tensor in zip(self.layers, self.caches.values()):
                columns[0].append(offset)
                columns[1].append(tensor.data_ptr())
                columns[2].append(tensor.stride(0) * tensor.element_size())
                columns[3].append(layer["bytes"] // 8)
                offset += layer["bytes"]
            self._tables = tuple(self.torch.tensor(c, dtype=self.torch.int64, device=self._device()) for c in columns)
        return self._tables

    def warm_up(self):
        """Build the tables and load every kernel once at registration, not on the first save or restore.

        Nothing is written to the KV cache: the gather reads block 0 into a
        scratch buffer, and the scatter runs gated shut.
        """
        torch = self.torch
        tables = self._load_tables()
        spans = self._spans()
        lib = _dp(self.pool.lib)
        device = self._device()
        with torch.cuda.stream(self._copy_stream):
            stream = self._copy_stream.cuda_stream
            scratch = torch.empty(self.block_bytes, dtype=torch.uint8, device=device)
            table = torch.tensor([0, scratch.data_ptr()], dtype=torch.int64, device=device)
            crc = torch.empty(1, dtype=torch.int32, device=device)
            digest = torch.empty(32, dtype=torch.uint8, device=device)
            gate = torch.ones(1, dtype=torch.int32, device=device)
            status = torch.zeros(1, dtype=torch.int32, device=device)
            calls = []
            for vec in sorted({self._span_vec, self._span_vec | self._hbm}):
                calls += [
                    lib.kvsnap_dp_gather(spans.data_ptr(), len(self.layers), self.block_bytes, table.data_ptr(),
                                         table.data_ptr() + 8, 1, 0, crc.data_ptr(), status.data_ptr(), vec,
                                         self.ctas, stream),
                    lib.kvsnap_dp_scatter(spans.data_ptr(), len(self.layers), self.block_bytes,
                                          table.data_ptr() + 8, table.data_ptr(), 1, 0, 0, gate.data_ptr(),
                                          status.data_ptr(), vec, self.ctas, stream),
                    lib.kvsnap_dp_crc32c(table.data_ptr() + 8, 1, self.block_bytes, crc.data_ptr(), 0,
                                         status.data_ptr(), vec, self.ctas, stream),
                ]
            calls.append(lib.kvsnap_dp_sha256(table.data_ptr() + 8, 1, self.block_bytes, digest.data_ptr(), stream))
            if min(calls) < 0:
                raise RuntimeError(lib.kvsnap_cuda_error().decode())
            empty = torch.zeros(1, dtype=torch.int64, device=device)
            copy_host_blocks(empty[:0], empty[:0], *tables)
        self._copy_stream.synchronize()
        if int(status.item()):
            raise RuntimeError(f"data-plane warm-up reported status {int(status.item())}")

    # ---- engine stream -----------------------------------------------------------------------

    def _validate_ids(self, ids):
        if getattr(self, "_min_blocks", None) is None:
            self._min_blocks = min(t.shape[0] for t in self.caches.values())
        limit = self._min_blocks
        for i in ids:
            if type(i) is not int or i < 0 or i >= limit:
                raise ValueError("GPU block id out of range")

    def producer_event(self):
        """A CUDA event recorded now on the engine's current stream."""
        event = self.torch.cuda.Event()
        event.record(self.torch.cuda.current_stream(self._device()))
        return event

    def wait_on_engine_stream(self, event):
        """Make the engine's current stream wait, on the GPU, for ``event``."""
        self.torch.cuda.current_stream(self._device()).wait_event(event)

    @contextmanager
    def staging(self, nblocks):
        """A packed pinned buffer for ``nblocks`` blocks, released (after its copies fence) on exit."""
        allocation = self.pool.reserve(self.block_bytes * nblocks)
        try:
            yield allocation
        finally:
            allocation.close()

    # ---- helpers ------------------------------------------------------------------------------

    def _vec_for(self, addresses):
        if self._span_vec == 16 and all(a % 16 == 0 for a in addresses):
            return 16
        if any(a % 8 for a in addresses):
            raise ValueError("packed blocks must be 8-byte aligned")
        return 8

    def _check(self, rc):
        if rc < 0:
            raise RuntimeError(self.pool.lib.kvsnap_cuda_error().decode())

    @staticmethod
    def _runs(endpoints, first, stop, size):
        """Runs [i, j) of consecutive blocks whose packed places are adjacent in one allocation."""
        i = first
        while i < stop:
            allocation, offset = endpoints[i]
            j = i + 1
            while j < stop and endpoints[j][0] is allocation and endpoints[j][1] == offset + (j - i) * size:
                j += 1
            yield i, j
            i = j

    def _status_error(self, status):
        value = int(status.item())
        if value & _abi.BAD_BLOCK:
            raise RuntimeError("data-plane kernel saw a block id outside its cache")
        if value & _abi.MISALIGNED:
            raise RuntimeError("data-plane kernel saw a misaligned address")
        if value & _abi.BAD_CUT:
            raise RuntimeError("data-plane kernel saw spans that do not pair or split as the flags asked")
        return value

    # ---- restore ------------------------------------------------------------------------------

    def load_scatter(self, block_ids, sources, *, progress=None, chunk_bytes=64 << 20, expected_crc32c=None,
                     cache=None, generations=None, known_digests=None):
        """Copy packed host blocks into ``block_ids`` and wait for it (reference dataplane.py:334-386).

        ``sources[i]`` is ``(allocation, offset)`` holding block i packed, in
        this pool's pinned memory. One scatter launch per ``chunk_bytes`` of
        blocks; a ``progress`` list receives ``(None, total bytes)`` and then, as
        each launch is queued, ``(its completion event, bytes left once it
        completes)``. Returns the number of launches.

        ``restore_mode`` "staged" (the default): per chunk, the copy engine moves
        the blocks into a two-slot device ring on the restore's copy stream and
        the scatter kernel writes them from there into the cache on the restore
        stream, chunk k+1's copy overlapping chunk k's scatter. "direct": the
        scatter kernel reads the pinned blocks in place. Both streams are the
        restore's own, so a restore overlaps a save's copies (the host link is
        full duplex).

        ``expected_crc32c``: the recorded CRC32C of each block. When given, all
        blocks are copied to device memory and checked there before any
        scatter is queued (and before ``progress`` is filled): a mismatch raises
        :class:`CorruptBlockError` with the KV cache untouched and no progress
        reported, so it stays a miss.

        ``cache`` (a :class:`DigestCache`), ``generations`` and
        ``known_digests``: the snapshot's ``(sha256 hex, crc32c)`` per block.
        Once the restore has completed, each block with a generation (not
        None) is recorded under it, so the next save of an unchanged block
        skips SHA-256.
        """
        torch = self.torch
        self._validate_ids(block_ids)
        if cache is not None and (generations is None or known_digests is None
                                  or len(generations) != len(block_ids) or len(known_digests) != len(block_ids)):
            raise ValueError("a digest cache needs one generation and one known digest per block")
        if len(sources) != len(block_ids):
            raise ValueError("one source per block is required")
        if expected_crc32c is not None and len(expected_crc32c) != len(block_ids):
            raise ValueError("one expected CRC32C per block is required")
        if not block_ids:
            return 0
        spans = self._spans()
        self._scatter_targets()
        lib = _dp(self.pool.lib)
        device = self._device()
        n, size = len(block_ids), self.block_bytes
        per_launch = max(1, chunk_bytes // size)
        verified = expected_crc32c is not None
        # Blocks of another process's shared arena (kvsnap_b200.sharedtier) are read in place.
        foreign = any(getattr(allocation, "foreign", False) for allocation, _ in sources)
        mode = "direct" if foreign else "staged" if verified else self.restore_mode
        copies, kernels = self._load_copy_stream, self._load_stream
        launches = 0
        done = None
        with self.pool.operation():
            # The pool lock keeps every source allocation open until the launches are queued.
            addresses = []
            for allocation, offset in sources:
                allocation._open()
                if offset < 0 or offset + size > allocation.size:
                    raise ValueError("load source outside its allocation")
                addresses.append(allocation.pointer + offset)
            with torch.cuda.stream(kernels):
                status = torch.zeros(1, dtype=torch.int32, device=device)
                ids = torch.tensor(list(block_ids), dtype=torch.int64).pin_memory().to(device, non_blocking=True)
                try:
                    if mode == "direct":
                        vec = self._vec_for(addresses)
                        table = torch.tensor(addresses, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
                        if verified:                 # every block checked where it lies, before any write
                            self._verify(table, n, expected_crc32c, status, vec, self.host_ctas)
                        if progress is not None:
                            progress.append((None, n * size))
                        for first in range(0, n, per_launch):
                            last = min(n, first + per_launch)
                            self._check(lib.kvsnap_dp_scatter(
                                spans.data_ptr(), len(self.layers), size, table[first:].data_ptr(),
                                ids[first:].data_ptr(), last - first, 0, 0, 0, status.data_ptr(), vec,
                                self.host_ctas, kernels.cuda_stream))
                            launches += 1
                            done = torch.cuda.Event()
                            done.record(kernels)
                            if progress is not None:
                                progress.append((done, (n - last) * size))
                        for allocation in {id(a): a for a, _ in sources}.values():
                            allocation.mark(kernels.cuda_stream)
                    elif verified and n * size > self.staging_bytes:
                        # Larger than the staging bound: check every block where it lies, then the chunk ring.
                        vec = self._vec_for(addresses)
                        table = torch.tensor(addresses, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
                        self._verify(table, n, expected_crc32c, status, vec, self.host_ctas)
                        launches, done = self._staged_chunks(sources, ids, n, per_launch, status, progress)
                    elif verified:
                        stage = torch.empty(n * size, dtype=torch.uint8, device=device)
                        stage.record_stream(copies)
                        base = stage.data_ptr()
                        self.pool.copy_many([(sources[i][0], sources[i][1], base + i * size, (j - i) * size)
                                             for i, j in self._runs(sources, 0, n, size)],
                                            to_host=False, stream=copies.cuda_stream)
                        landed = torch.cuda.Event()
                        landed.record(copies)
                        kernels.wait_event(landed)
                        vec = (16 | self._hbm) if size % 16 == 0 else 8
                        table = torch.tensor([base + i * size for i in range(n)], dtype=torch.int64).pin_memory().to(
                            device, non_blocking=True)
                        self._verify(table, n, expected_crc32c, status, vec)
                        if progress is not None:
                            progress.append((None, n * size))
                        for first in range(0, n, per_launch):
                            last = min(n, first + per_launch)
                            self._check(lib.kvsnap_dp_scatter(
                                spans.data_ptr(), len(self.layers), size, table[first:].data_ptr(),
                                ids[first:].data_ptr(), last - first, 0, 0, 0, status.data_ptr(), vec, self.hbm_ctas,
                                kernels.cuda_stream))
                            launches += 1
                            done = torch.cuda.Event()
                            done.record(kernels)
                            if progress is not None:
                                progress.append((done, (n - last) * size))
                    else:
                        launches, done = self._staged_chunks(sources, ids, n, per_launch, status, progress)
                except BaseException:
                    # A launch or copy that failed part way may still be queued:
                    # nothing may release the sources before both streams drain.
                    copies.synchronize()
                    kernels.synchronize()
                    raise
        done.synchronize()
        self._status_error(status)
        if cache is not None:
            for block, generation, digest in zip(block_ids, generations, known_digests):
                if generation is not None:
                    cache.put(block, generation, digest)
        return launches

    def _staged_chunks(self, sources, ids, n, per_launch, status, progress):
        """Restore through a two-slot device ring: copy engine in, scatter kernel out, per chunk."""
        torch = self.torch
        lib = _dp(self.pool.lib)
        spans = self._spans()
        device = self._device()
        size = self.block_bytes
        copies, kernels = self._load_copy_stream, self._load_stream
        depth = min(n, per_launch)
        ring = torch.empty(2 * depth * size, dtype=torch.uint8, device=device)
        ring.record_stream(copies)
        base = ring.data_ptr()
        table = torch.tensor([base + i * size for i in range(2 * depth)], dtype=torch.int64).pin_memory().to(
            device, non_blocking=True)
        vec = (16 | self._hbm) if size % 16 == 0 else 8
        if progress is not None:
            progress.append((None, n * size))
        scattered, done, launches = [], None, 0
        for chunk, first in enumerate(range(0, n, per_launch)):
            last = min(n, first + per_launch)
            slot = chunk % 2
            if chunk >= 2:
                copies.wait_event(scattered[chunk - 2])      # the slot's previous chunk is in the cache
            self.pool.copy_many([(sources[i][0], sources[i][1], base + (slot * depth + i - first) * size,
                                  (j - i) * size) for i, j in self._runs(sources, first, last, size)],
                                to_host=False, stream=copies.cuda_stream)
            landed = torch.cuda.Event()
            landed.record(copies)
            kernels.wait_event(landed)
            self._check(lib.kvsnap_dp_scatter(
                spans.data_ptr(), len(self.layers), size, table[slot * depth:].data_ptr(), ids[first:].data_ptr(),
                last - first, 0, 0, 0, status.data_ptr(), vec, self.hbm_ctas, kernels.cuda_stream))
            launches += 1
            done = torch.cuda.Event()
            done.record(kernels)
            scattered.append(done)
            if progress is not None:
                progress.append((done, (n - last) * size))
        return launches, done

    def _verify(self, table, n, expected, status, vec, ctas=None):
        """CRC32C of the blocks at table[:n] (device staging, or pinned memory read over the host link) against
        ``expected``; raises before any scatter is queued."""
        torch = self.torch
        lib = _dp(self.pool.lib)
        crc = torch.empty(n, dtype=torch.int32, device=table.device)
        expect = torch.tensor(_u32(expected), dtype=torch.int32).pin_memory().to(table.device, non_blocking=True)
        self._check(lib.kvsnap_dp_crc32c(table.data_ptr(), n, self.block_bytes, crc.data_ptr(), expect.data_ptr(),
                                         status.data_ptr(), vec, self.hbm_ctas if ctas is None else ctas,
                                         torch.cuda.current_stream().cuda_stream))
        flags = int(status.item())          # synchronises the copy stream
        if flags & _abi.CRC_MISMATCH:
            got = [v & 0xFFFFFFFF for v in crc.tolist()]
            bad = [i for i, (g, e) in enumerate(zip(got, expected)) if g != e]
            raise CorruptBlockError(f"packed block checksum mismatch at block index {bad[0]}", bad)
        if flags:
            self._status_error(status)

    # ---- save ---------------------------------------------------------------------------------

    def save_gather(self, block_ids, targets, num_kv_tokens, *, chunk_bytes=64 << 20, digests=None,
                    cache=None, generations=None):
        """Gather blocks on the GPU and land them packed in pinned memory (reference dataplane.py:388-437).

        ``targets[i]`` is ``(allocation, offset)`` receiving block i packed, the
        layout :meth:`load_scatter` reads. The caller must have fenced the
        producer stream. Token slots past ``num_kv_tokens`` in the last block
        are written as zeros, so a snapshot never carries stale KV. Returns the
        number of device-to-host copies (staged mode: one per run of adjacent
        targets in one allocation, per ``chunk_bytes`` of blocks) or of kernel
        launches (direct mode; and, above ``staging_bytes``, the column
        landings).

        ``digests``: a list that receives ``(sha256 hex, crc32c)`` for each
        packed block, the store's content id and checksum, computed on the GPU
        from the same bytes the targets receive. A :class:`PendingDigests`
        instead returns as soon as the targets are written (the point at which
        the connector may free the GPU blocks) while the SHA-256 kernel still
        runs; its ``result()`` waits for it and returns the list. The targets
        must stay allocated until then.

        ``cache`` (a :class:`DigestCache`) with ``generations[i]`` for each
        block: full blocks found in the cache are not hashed again (their
        CRC32C, computed by the gather anyway, must equal the cached one), and
        every full block's digest is stored for the next save.

        Device staging is bounded by ``staging_bytes``: a session that does not
        fit moves through a ring of device slots a column (a run of spans of
        every block) at a time, the SHA-256 of each block carried from column
        to column.
        """
        torch = self.torch
        self._validate_ids(block_ids)
        expected = (num_kv_tokens + self.block_size - 1) // self.block_size
        if len(block_ids) != expected or len(targets) != len(block_ids):
            raise ValueError("block count does not cover computed tokens")
        if not block_ids:
            return 0
        if (cache is None) != (generations is None):
            raise ValueError("a digest cache needs one generation per block, and generations a cache")
        if generations is not None and len(generations) != len(block_ids):
            raise ValueError("one generation per block is required")
        if cache is not None and digests is None:
            raise ValueError("a digest cache serves digests: pass digests= as well")
        spans = self._spans()
        stream = self._scatter_targets()
        n, size = len(block_ids), self.block_bytes
        valid = num_kv_tokens % self.block_size
        # Full blocks only: the last block's tail slots are zeroed and change with the next token.
        full = n if valid == 0 else n - 1
        known = {}
        if cache is not None:
            for i in range(full):
                entry = cache.get(block_ids[i], generations[i])
                if entry is not None:
                    known[i] = entry
        job = _SaveJob(block_ids, targets, valid, [i for i in range(n) if i not in known], known, digests is not None)
        with torch.cuda.stream(stream):
            job.status = torch.zeros(1, dtype=torch.int32, device=self._device())
            job.crc = torch.zeros(n, dtype=torch.int32, device=self._device()) if job.digests else None
            try:
                if self.save_mode == "direct" and not job.digests:
                    copies = self._save_direct(job, spans, chunk_bytes)
                elif n * size <= self.staging_bytes or self._span_vec != 16:
                    copies = self._save_whole(job, spans, chunk_bytes)
                else:
                    copies = self._save_columns(job)
                done = torch.cuda.Event()
                done.record()
            except BaseException:
                stream.synchronize()
                for other in (job.side, job.land):
                    if other is not None:
                        other.synchronize()
                raise
        done.synchronize()
        self.pool.wait_many({id(a): a for a, _ in targets}.values())
        self._status_error(job.status)
        if job.digests:
            finished = torch.cuda.Event()
            finished.record(job.side)
            pending = digests if isinstance(digests, PendingDigests) else PendingDigests()
            keys = [(block_ids[i], generations[i]) for i in range(full)] if cache is not None else []
            pending._bind(finished, lambda: self._digests(job, cache, keys))
            if not isinstance(digests, PendingDigests):
                digests.extend(pending.result())
        return copies

    def _save_direct(self, job, spans, chunk_bytes):
        """The gather kernel writes the pinned targets in place over the host link."""
        torch = self.torch
        lib = _dp(self.pool.lib)
        stream = self._copy_stream
        n, size = len(job.block_ids), self.block_bytes
        for allocation, offset in job.targets:
            allocation._open()
            if offset < 0 or offset + size > allocation.size:
                raise ValueError("save target outside its allocation")
        write_to = [a.pointer + o for a, o in job.targets]
        vec = self._vec_for(write_to)
        table = torch.tensor(list(job.block_ids) + write_to, dtype=torch.int64).pin_memory().to(
            self._device(), non_blocking=True)
        per_chunk = max(1, min(n, chunk_bytes // size))
        launches = 0
        for first in range(0, n, per_chunk):
            last = min(n, first + per_chunk)
            self._check(lib.kvsnap_dp_gather(
                spans.data_ptr(), len(self.layers), size, table[first:].data_ptr(), table[n + first:].data_ptr(),
                last - first, job.valid if last == n else 0, 0, job.status.data_ptr(), vec, self.host_ctas,
                stream.cuda_stream))
            launches += 1
        for allocation in {id(a): a for a, _ in job.targets}.values():
            allocation.mark()
        return launches

    def _save_whole(self, job, spans, chunk_bytes):
        """Every block gathered into device staging at once; the copy engine lands it, SHA-256 reads it in place."""
        torch = self.torch
        lib = _dp(self.pool.lib)
        stream = self._copy_stream
        n, size = len(job.block_ids), self.block_bytes
        stage = torch.empty(n * size, dtype=torch.uint8, device=self._device())
        write_to = [stage.data_ptr() + i * size for i in range(n)]
        vec = self._vec_for(write_to)
        if vec == 16:
            vec |= self._hbm
        table = torch.tensor(list(job.block_ids) + write_to, dtype=torch.int64).pin_memory().to(
            self._device(), non_blocking=True)
        self._check(lib.kvsnap_dp_gather(
            spans.data_ptr(), len(self.layers), size, table.data_ptr(), table[n:].data_ptr(), n, job.valid,
            job.crc.data_ptr() if job.crc is not None else 0, job.status.data_ptr(), vec, self.hbm_ctas,
            stream.cuda_stream))
        if job.digests:
            job.side = self._sha_stream()
            addresses = table[n:] if len(job.hashed) == n else torch.tensor(
                [write_to[i] for i in job.hashed], dtype=torch.int64).pin_memory().to(self._device(), non_blocking=True)
            job.digest = self._sha256_after(stage, addresses, len(job.hashed), stream, job.side)
        job.keep = stage
        job.rehash_from = write_to
        per_chunk = max(1, min(n, chunk_bytes // size))
        entries = []
        for first in range(0, n, per_chunk):
            for i, j in self._runs(job.targets, first, min(n, first + per_chunk), size):
                allocation, offset = job.targets[i]
                entries.append((allocation, offset, stage.data_ptr() + i * size, (j - i) * size))
        self.pool.copy_many(entries, to_host=True)
        return len(entries)

    def _save_columns(self, job):
        """A save larger than ``staging_bytes``: a ring of device slots, one column of a group of blocks a slot.

        For each (group, column): the gather writes the column of every block
        of the group into a free slot (CRC shares accumulate per block), the
        column lands at each target's column offset in pinned memory, and the
        SHA-256 kernel advances every block's hash over it from the state the
        previous column left. A landing kernel stores the column (one copy a
        block piece would be too small for the copy engine to run at the link
        rate); with ``column_landing="copy"`` and a group whose targets lie at
        one pitch, the column lands as one copy-engine transfer on the landing
        stream while the SMs gather the next column.
        A slot is reused once it has landed and its hash part is done, so
        device memory stays within ``staging_bytes`` while all blocks hash at
        once. Needs 16-byte aligned spans and targets (the CRC shares of the
        segment kernels accumulate across calls; the landing stores are 16
        bytes).
        """
        torch = self.torch
        lib = _dp(self.pool.lib)
        stream = self._copy_stream
        device = self._device()
        n, size = len(job.block_ids), self.block_bytes
        slots = self.staging_slots
        group, stride, columns, tables, flags = self._columns(n)
        slot_bytes = group * stride
        with self.pool.operation():
            # The pool lock keeps every target open until the kernels writing it are fenced under it.
            for allocation, offset in job.targets:
                allocation._open()
                if offset < 0 or offset + size > allocation.size:
                    raise RuntimeError("copy outside pinned allocation")
            targets = [a.pointer + o for a, o in job.targets]
            if any(t % 16 for t in targets):
                raise ValueError("packed blocks must be 16-byte aligned for a bounded save")
            ring = torch.empty(slots * slot_bytes, dtype=torch.uint8, device=device)
            base = ring.data_ptr()
            groups = [(g0, min(n, g0 + group)) for g0 in range(0, n, group)]
            pitches = [_even_pitch(targets, g0, g1, size) if self.column_landing == "copy" else None
                       for g0, g1 in groups]
            if any(p is not None for p in pitches):
                job.land = self._land_stream
                ring.record_stream(job.land)
            hashed_in = [[i for i in job.hashed if g0 <= i < g1] for g0, g1 in groups]
            # One upload: block ids, target addresses, each slot's block addresses, and for a group whose
            # blocks are not all hashed, per slot the addresses of those that are.
            host = list(job.block_ids) + targets
            slot_at = len(host)
            host += [base + r * slot_bytes + k * stride for r in range(slots) for k in range(group)]
            own_table = {}
            if job.digests:
                for g, (g0, g1) in enumerate(groups):
                    if hashed_in[g] and hashed_in[g] != list(range(g0, g1)):
                        for r in range(slots):
                            own_table[g, r] = len(host)
                            host += [base + r * slot_bytes + (i - g0) * stride for i in hashed_in[g]]
            table = torch.tensor(host, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
            words = table.data_ptr()
            state = None
            if job.digests:
                job.side = self._sha_stream()
                ring.record_stream(job.side)
                table.record_stream(job.side)
                # The hash parts write these on the side stream after this call returns: allocated there, and
                # held by the job until its digests are read, so no other allocation can take them meanwhile.
                with torch.cuda.stream(job.side):
                    job.digest = torch.empty(max(1, len(job.hashed)) * 32, dtype=torch.uint8, device=device)
                    state = torch.empty(max(1, len(job.hashed)) * 8, dtype=torch.int32, device=device)
            launches, hashed_before, unit = 0, 0, 0
            read = []          # per unit: the event after which its slot's hash part is done, or None
            landed = []        # per unit: the event after which the landing stream has moved its slot, or None
            for g, (g0, g1) in enumerate(groups):
                for j, (s0, s1, offset, nbytes) in enumerate(columns):
                    r = unit % slots
                    slot = base + r * slot_bytes
                    slot_table = words + 8 * (slot_at + r * group)
                    if unit >= slots:
                        for before in (read[unit - slots], landed[unit - slots]):
                            if before is not None:
                                stream.wait_event(before)
                    self._check(lib.kvsnap_dp_gather(
                        tables[j].data_ptr(), s1 - s0, size, words + 8 * g0, slot_table, g1 - g0,
                        job.valid if g1 == n else 0, job.crc.data_ptr() + 4 * g0 if job.crc is not None else 0,
                        job.status.data_ptr(), flags[j], self._grid_beside(len(job.hashed)), stream.cuda_stream))
                    gathered = None
                    if pitches[g] is not None:
                        gathered = torch.cuda.Event()
                        gathered.record(stream)
                        job.land.wait_event(gathered)
                        self._check(lib.kvsnap_dp_land_strided(slot, stride, targets[g0] + offset, pitches[g],
                                                               g1 - g0, nbytes, job.land.cuda_stream))
                        moved = torch.cuda.Event()
                        moved.record(job.land)
                        landed.append(moved)
                    else:
                        self._check(lib.kvsnap_dp_land(slot, stride, words + 8 * (n + g0), offset, g1 - g0, nbytes,
                                                       job.status.data_ptr(), 0, stream.cuda_stream))
                        landed.append(None)
                    launches += 1
                    event = None
                    if job.digests and hashed_in[g]:
                        if gathered is None:
                            gathered = torch.cuda.Event()
                            gathered.record(stream)
                        job.side.wait_event(gathered)
                        at = words + 8 * own_table[g, r] if (g, r) in own_table else slot_table
                        last = j == len(columns) - 1
                        self._check(lib.kvsnap_dp_sha256_part(
                            at, len(hashed_in[g]), nbytes, offset, size, state.data_ptr() + 32 * hashed_before,
                            job.digest.data_ptr() + 32 * hashed_before if last else 0, job.side.cuda_stream))
                        event = torch.cuda.Event()
                        event.record(job.side)
                    read.append(event)
                    unit += 1
                hashed_before += len(hashed_in[g])
            if job.land is not None:
                last = torch.cuda.Event()
                last.record(job.land)
                stream.wait_event(last)                  # the targets are written once the copy stream passes here
            if job.crc is not None:
                self._check(lib.kvsnap_dp_crc32c_finish(job.crc.data_ptr(), 0, n, size, job.status.data_ptr(),
                                                        stream.cuda_stream))
            for allocation in {id(a): a for a, _ in job.targets}.values():
                allocation.mark()
        job.keep = (ring, table, state)
        job.rehash_from = targets
        return launches

    def _columns(self, n):
        """The column plan for saves of n blocks, with each column's device span table and kernel flags."""
        plans = self.__dict__.setdefault("_column_plans", {})
        if n not in plans:
            span_bytes = [layer["bytes"] for layer in self.layers]
            group, stride, columns = column_plan(span_bytes, n, self.staging_bytes // self.staging_slots)
            host = (_abi.Span * len(self.layers)).from_buffer_copy(self._span_table.cpu().numpy().tobytes())
            tables, flags = [], []
            for s0, s1, offset, _ in columns:
                part = (_abi.Span * (s1 - s0))()
                for k in range(s1 - s0):
                    part[k] = host[s0 + k]
                    part[k].offset -= offset                 # packed offsets from the column's start
                tables.append(self.torch.frombuffer(bytearray(bytes(part)), dtype=self.torch.uint8).to(self._device()))
                vec = 16 if self._span_vec == 16 and stride % 16 == 0 else 8
                flags.append(vec | (_abi.hbm_flags(span_bytes[s0:s1], vec) | _abi.CRC_ACCUMULATE if vec == 16 else 0))
            plans[n] = (group, stride, columns, tables, flags)
        return plans[n]

    def _digests(self, job, cache, keys):
        """The save's ``(sha256 hex, crc32c)`` list, once its SHA-256 kernels have finished.

        Blocks served from ``cache`` must have kept their CRC32C; one that has
        not is hashed now, from wherever the save left its packed bytes
        (device staging, or the pinned targets).
        """
        torch = self.torch
        crcs = [v & 0xFFFFFFFF for v in job.crc.cpu().tolist()]
        raw = job.digest.cpu().numpy().tobytes() if job.hashed else b""
        out = [None] * len(crcs)
        for k, i in enumerate(job.hashed):
            out[i] = (raw[32 * k:32 * k + 32].hex(), crcs[i])
        stale = [i for i, (sha, c) in job.known.items() if c != crcs[i]]
        for i, entry in job.known.items():
            out[i] = (entry[0], crcs[i])
        if cache is not None:
            cache.hits += len(job.known) - len(stale)
            cache.misses += len(keys) - len(job.known)
            cache.rejected += len(stale)
        if stale:
            lib = _dp(self.pool.lib)
            stream = self._sha_stream()
            device = self._device()
            with torch.cuda.stream(stream):
                addresses = torch.tensor([job.rehash_from[i] for i in stale], dtype=torch.int64, device=device)
                fresh = torch.empty(len(stale) * 32, dtype=torch.uint8, device=device)
                self._check(lib.kvsnap_dp_sha256(addresses.data_ptr(), len(stale), self.block_bytes,
                                                 fresh.data_ptr(), stream.cuda_stream))
            stream.synchronize()
            raw = fresh.cpu().numpy().tobytes()
            for k, i in enumerate(stale):
                out[i] = (raw[32 * k:32 * k + 32].hex(), crcs[i])
        if cache is not None:
            for i, key in enumerate(keys):
                cache.put(key[0], key[1], out[i])
        job.keep = None
        return out

    def _sha_stream(self):
        with self._sha_lock:
            side = self._sha_streams[self._sha_next % len(self._sha_streams)]
            self._sha_next += 1
        return side

    def _sha256_after(self, stage, addresses, n, stream, side):
        """SHA-256 of the staged blocks on ``side``, after the work queued on ``stream`` so far."""
        torch = self.torch
        lib = _dp(self.pool.lib)
        ready = torch.cuda.Event()
        ready.record(stream)
        side.wait_event(ready)
        with torch.cuda.stream(side):
            out = torch.empty(n * 32, dtype=torch.uint8, device=addresses.device)
            self._check(lib.kvsnap_dp_sha256(addresses.data_ptr(), n, self.block_bytes, out.data_ptr(),
                                             side.cuda_stream))
        # The staging buffer and tables belong to the copy stream's allocator pool;
        # keep them from reuse until the side stream is done with them.
        stage.record_stream(side)
        addresses.record_stream(side)
        return out

    # ---- checksums of blocks already in pinned memory ---------------------------------------------

    def digest(self, sources):
        """``(sha256 hex, crc32c)`` of packed blocks in pinned memory, computed on the GPU.

        ``sources[i]`` is ``(allocation, offset)``; each block is copied to
        device memory by the copy engine and hashed there. The values of the
        reference's host ``_digest`` (kvsnap/connector/volatile.py:141-151).
        """
        torch = self.torch
        if not sources:
            return []
        self._spans()
        stream = self._scatter_targets()
        lib = _dp(self.pool.lib)
        device = self._device()
        n, size = len(sources), self.block_bytes
        with self.pool.operation():
            for allocation, offset in sources:
                allocation._open()
                if offset < 0 or offset + size > allocation.size:
                    raise ValueError("digest source outside its allocation")
            with torch.cuda.stream(stream):
                if n * size <= self.staging_bytes:
                    stage = torch.empty(n * size, dtype=torch.uint8, device=device)
                    self.pool.copy_many([(sources[i][0], sources[i][1], stage.data_ptr() + i * size, (j - i) * size)
                                         for i, j in self._runs(sources, 0, n, size)], to_host=False)
                    where = [stage.data_ptr() + i * size for i in range(n)]
                    vec, ctas = ((16 | _abi.HBM) if size % 16 == 0 else 8), self.hbm_ctas
                else:
                    # Beyond the staging bound the kernels read the pinned blocks in place over the host link.
                    where = [a.pointer + o for a, o in sources]
                    vec, ctas = self._vec_for(where), self.host_ctas
                addresses = torch.tensor(where, dtype=torch.int64).pin_memory().to(device, non_blocking=True)
                crc = torch.empty(n, dtype=torch.int32, device=device)
                status = torch.zeros(1, dtype=torch.int32, device=device)
                out = torch.empty(n * 32, dtype=torch.uint8, device=device)
                self._check(lib.kvsnap_dp_crc32c(addresses.data_ptr(), n, size, crc.data_ptr(), 0,
                                                 status.data_ptr(), vec, ctas, stream.cuda_stream))
                self._check(lib.kvsnap_dp_sha256(addresses.data_ptr(), n, size, out.data_ptr(), stream.cuda_stream))
            stream.synchronize()
        self._status_error(status)
        crcs = [v & 0xFFFFFFFF for v in crc.cpu().tolist()]
        raw = out.cpu().numpy().tobytes()
        return [(raw[32 * i:32 * i + 32].hex(), crcs[i]) for i in range(n)]

    def close(self):
        self.pool.close()
