"""Native host CRC32C and blob file I/O: a drop-in for kvsnap's ``kvsnap.store.native_io`` native backend.

``NativeIO`` binds ``_io_native.so`` (include/kvsnap_io.h) with the same
methods, argument checks and errors as the reference's NativeIO
(kvsnap/store/native_io.py:51-151): ``pwrite_all``, ``pread_all``,
``pread_into``, ``crc32c``, ``crc32c_at``, ``close``. ``get_io_backend`` returns
the process-wide instance (reopened after fork). There is no pure-Python
backend here: a missing library raises.
"""
from __future__ import annotations

import atexit
import ctypes as C
import os
import threading
from pathlib import Path

from . import _abi

_NATIVE = Path(__file__).resolve().parent / "_native"


class NativeIO:
    name = "native"

    def __init__(self, path, *, workers=2, queue_bytes=64 * 1024**2):
        self.lib = _abi.load(path, _abi.IO_API)
        if self.lib.kvsnap_io_abi_version() != _abi.IO_ABI_VERSION:
            raise RuntimeError("unsupported kvsnap native I/O ABI")
        if type(workers) is not int or not 1 <= workers <= 64 or type(queue_bytes) is not int or queue_bytes <= 0:
            raise ValueError("invalid native I/O capacity")
        self.handle = self.lib.kvsnap_io_pool_create(workers, queue_bytes)
        if not self.handle:
            raise RuntimeError("native I/O pool creation failed")
        self.queue_bytes = queue_bytes
        self.pid = os.getpid()
        self._lifecycle = threading.Condition()
        self._active = 0
        self._closing = False
        atexit.register(self.close)

    def _open(self):
        if self.pid != os.getpid():
            raise RuntimeError("native I/O pools must be reopened after fork")
        if not self.handle or self._closing:
            raise RuntimeError("native I/O pool is closed")

    @staticmethod
    def _offset(size, offset):
        if type(size) is not int or type(offset) is not int or min(size, offset) < 0 or size + offset > 2**63 - 1:
            raise ValueError("invalid I/O range")

    def _transfer(self, fd, data, size, offset, write):
        self._offset(size, offset)
        if self.pid != os.getpid():
            raise RuntimeError("native I/O pools must be reopened after fork")
        with self._lifecycle:
            self._open()
            self._active += 1
        try:
            code = self.lib.kvsnap_io_pool_transfer(self.handle, fd, data, size, offset, write, 0)
        finally:
            with self._lifecycle:
                self._active -= 1
                self._lifecycle.notify_all()
        if code:
            raise OSError(code, os.strerror(code))

    def pwrite_all(self, fd, data, offset):
        data = bytes(data)
        self._offset(len(data), offset)
        # Bounded pieces, so one transfer never exceeds the pool's byte budget.
        for index in range(0, len(data), self.queue_bytes):
            part = data[index:index + self.queue_bytes]
            self._transfer(fd, C.c_char_p(part), len(part), offset + index, 1)

    def pread_all(self, fd, size, offset):
        self._offset(size, offset)
        result = C.create_string_buffer(size)
        for index in range(0, size, self.queue_bytes):
            count = min(self.queue_bytes, size - index)
            self._transfer(fd, C.byref(result, index), count, offset + index, 0)
        return result.raw

    def pread_into(self, fd, address, size, offset):
        """Read straight into caller memory (e.g. pinned host memory), no Python copy."""
        self._offset(size, offset)
        for index in range(0, size, self.queue_bytes):
            count = min(self.queue_bytes, size - index)
            self._transfer(fd, C.c_void_p(address + index), count, offset + index, 0)

    def pwrite_from(self, fd, address, size, offset):
        """Write straight from caller memory (e.g. pinned host memory), no Python copy."""
        self._offset(size, offset)
        for index in range(0, size, self.queue_bytes):
            count = min(self.queue_bytes, size - index)
            self._transfer(fd, C.c_void_p(address + index), count, offset + index, 1)

    def crc32c(self, data, crc=0):
        self._open()
        data = bytes(data)
        return int(self.lib.kvsnap_crc32c_extend(C.c_char_p(data), len(data), crc))

    def crc32c_at(self, address, size, crc=0):
        self._open()
        return int(self.lib.kvsnap_crc32c_extend(C.c_void_p(address), size, crc))

    def close(self):
        if self.pid != os.getpid():
            return
        with self._lifecycle:
            if not self.handle:
                return
            self._closing = True
            self._lifecycle.wait_for(lambda: self._active == 0)
            self.lib.kvsnap_io_pool_destroy(self.handle)
            self.handle = None


_backends = {}
_cache_lock = threading.Lock()


def _after_fork():
    global _backends, _cache_lock
    # The parent's pools have no worker threads in the child; open new ones lazily.
    _backends = {}
    _cache_lock = threading.Lock()


if hasattr(os, "register_at_fork"):
    os.register_at_fork(after_in_child=_after_fork)


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
    key = (os.getpid(), str(path.resolve()))
    with _cache_lock:
        if key not in _backends:
            _backends[key] = NativeIO(path)
        return _backends[key]
