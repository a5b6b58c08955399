"""Native host CRC32C and blob file I/O: a drop-in for kvsnap's ``kvsnap.store.native_io`` native backend.

``NativeIO`` binds ``_io_native.so`` (include/kvsnap_io.h) with the methods,
argument checks and errors of the reference's NativeIO
(kvsnap/store/native_io.py:51-151): ``pwrite_all``, ``pread_all``,
``pread_into``, ``crc32c``, ``crc32c_at``, ``close``, plus ``pwrite_from``
for writes straight out of pinned memory. ``get_io_backend`` returns the
process-wide instance for the library (a fresh one after fork). There is no
pure-Python backend here: a missing library raises.
"""
from __future__ import annotations

import atexit
import ctypes as C
import os
import threading
from contextlib import contextmanager
from pathlib import Path

from . import _abi

_NATIVE = Path(__file__).resolve().parent / "_native"
_MAX_OFFSET = 2**63 - 1


def _check_range(size, offset):
    """A transfer of ``size`` bytes at ``offset``: non-negative ints that stay inside a 63-bit file offset."""
    if type(size) is not int or type(offset) is not int or size < 0 or offset < 0 or size + offset > _MAX_OFFSET:
        raise ValueError("invalid I/O range")


class _InFlight:
    """Counts calls inside the native pool, so that a close can wait for the last one to return."""

    def __init__(self):
        self._changed = threading.Condition()
        self._count = 0
        self.closing = False

    @contextmanager
    def call(self, may_start):
        with self._changed:
            may_start()
            self._count += 1
        try:
            yield
        finally:
            with self._changed:
                self._count -= 1
                if self._count == 0:
                    self._changed.notify_all()

    def drain(self):
        """Refuse new calls, then wait until none is running."""
        with self._changed:
            self.closing = True
            self._changed.wait_for(lambda: self._count == 0)


class NativeIO:
    """Blob-file transfers through the native transfer pool and CRC32C over host memory.

    Transfers larger than the pool's byte budget go through in budget-sized
    pieces, each a positional read or write of its own, from the caller's
    buffer in place.
    """

    name = "native"

    def __init__(self, path, *, workers=2, queue_bytes=64 * 1024**2):
        lib = _abi.load(path, _abi.IO_API)
        if lib.kvsnap_io_abi_version() != _abi.IO_ABI_VERSION:
            raise RuntimeError("unsupported kvsnap native I/O ABI")
        if type(workers) is not int or type(queue_bytes) is not int or not (1 <= workers <= 64 and queue_bytes > 0):
            raise ValueError("invalid native I/O capacity")
        handle = lib.kvsnap_io_pool_create(workers, queue_bytes)
        if not handle:
            raise RuntimeError("native I/O pool creation failed")
        self.lib, self.handle, self.queue_bytes = lib, handle, queue_bytes
        self.pid = os.getpid()
        self._calls = _InFlight()
        atexit.register(self.close)

    def _usable(self):
        if self.pid != os.getpid():
            raise RuntimeError("native I/O pools must be reopened after fork")
        if not self.handle or self._calls.closing:
            raise RuntimeError("native I/O pool is closed")

    def _move(self, fd, address, size, offset, write):
        """``size`` bytes between ``address`` and the file at ``offset``, in pieces of at most the pool's budget."""
        _check_range(size, offset)
        with self._calls.call(self._usable):
            for done in range(0, size, self.queue_bytes):
                piece = min(self.queue_bytes, size - done)
                code = self.lib.kvsnap_io_pool_transfer(self.handle, fd, address + done, piece, offset + done,
                                                        int(write), 0)
                if code:
                    raise OSError(code, os.strerror(code))

    def pwrite_all(self, fd, data, offset):
        payload = data if isinstance(data, bytes) else bytes(data)
        _check_range(len(payload), offset)
        address = C.cast(C.c_char_p(payload), C.c_void_p).value or 0
        self._move(fd, address, len(payload), offset, True)

    def pread_all(self, fd, size, offset):
        _check_range(size, offset)
        result = C.create_string_buffer(size)
        self._move(fd, C.addressof(result), size, offset, False)
        return result.raw

    def pread_into(self, fd, address, size, offset):
        """Read straight into caller memory (e.g. pinned host memory), no Python copy."""
        self._move(fd, address, size, offset, False)

    def pwrite_from(self, fd, address, size, offset):
        """Write straight from caller memory (e.g. pinned host memory), no Python copy."""
        self._move(fd, address, size, offset, True)

    def crc32c(self, data, crc=0):
        self._usable()
        payload = data if isinstance(data, bytes) else bytes(data)
        return int(self.lib.kvsnap_crc32c_extend(C.c_char_p(payload), len(payload), crc))

    def crc32c_at(self, address, size, crc=0):
        self._usable()
        return int(self.lib.kvsnap_crc32c_extend(C.c_void_p(address), size, crc))

    def close(self):
        """Refuse new transfers, wait for running ones, then free the native pool (no-op in a forked child)."""
        if self.pid != os.getpid() or not self.handle:
            return
        self._calls.drain()
        handle, self.handle = self.handle, None
        if handle:
            self.lib.kvsnap_io_pool_destroy(handle)


class _Backends:
    """One NativeIO per (process, library path)."""

    def __init__(self):
        self.lock = threading.Lock()
        self.by_key = {}

    def get(self, path):
        key = (os.getpid(), str(path.resolve()))
        with self.lock:
            backend = self.by_key.get(key)
            if backend is None:
                backend = self.by_key[key] = NativeIO(path)
            return backend


_registry = _Backends()


def _forget_parent_backends():
    # A forked child inherits the parent's pools without their callers; it opens its own on first use.
    global _registry
    _registry = _Backends()


if hasattr(os, "register_at_fork"):
    os.register_at_fork(after_in_child=_forget_parent_backends)


def resolve_io_library():
    override = os.environ.get("KVSNAP_IO_LIBRARY")
    if override:
        return Path(override)
    found = sorted(_NATIVE.glob("_io_native*.so"))
    return found[0] if found else _NATIVE / "_io_native.so"


def get_io_backend(mode=None):
    """The native I/O backend (reference native_io.py:170-190, native and auto modes)."""
    mode = mode or os.environ.get("KVSNAP_IO_BACKEND", "auto")
    if mode not in ("auto", "native"):
        raise ValueError("KVSNAP_IO_BACKEND must be auto or native")
    path = resolve_io_library()
    if not path.is_file():
        raise RuntimeError(f"native I/O library missing at {path}; build it with python -m kvsnap_b200.build")
    return _registry.get(path)
