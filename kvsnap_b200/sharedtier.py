"""The host tier across worker processes: another owner's pinned blocks read in place.

In kvsnap, a host-tier ("volatile") snapshot lives in the pinned memory of the
worker that saved it. A worker that restores a snapshot another live worker
owns fetches every block from that owner over a Unix socket, checks its
CRC32C on the host and copies it into local pinned staging before the
restore (kvsnap/connector/vllm.py:524-534 over connector/volatile.py:87-138,
``VolatileClient.read``).

Here the owner's pinned pool is POSIX shared memory
(``CudaPool(..., shared_name=new_segment_name())``): the same pool, whose
arena other processes of the same user can map. The owner hands out, per
block, a location ``{"segment": name, "offset": bytes into the arena,
"length": block bytes}`` (``locations``). A restoring worker maps the segment
read-only, registers it with its own CUDA context (``SharedBlocks``) and passes
``sources(...)`` straight to ``TorchBlockDataPlane.load_scatter``: the restore
kernel reads the owner's bytes in place over the host link, and with
``expected_crc32c=`` every block is checked on the GPU before any KV byte is
written. No bytes go through a socket, a Python buffer or a host copy.

Access: the segment is created with mode 0600 under an unguessable name (128
random bits), so only processes of the owner's user that were told the name
can map it, and they map it read-only. Lifetime: the owner unlinks the name
when its pool closes; a mapping made before that stays valid until its
``SharedBlocks`` closes, which first waits for the kernels that read it. Which
blocks an owner still holds, and the leases that keep them, stay the
control plane's business (the reference's owner protocol), as they are for
the socket path.
"""
from __future__ import annotations

import ctypes as C
import os
import secrets
import threading


def new_segment_name() -> str:
    """A fresh shared-memory name: one path component, 128 random bits."""
    return "/kvsnap-" + secrets.token_hex(16)


def locations(pool, allocations):
    """Where each of ``allocations`` (in the shared ``pool``) lies, for a worker in another process."""
    if pool.shared_name is None:
        raise ValueError("locations name a shared pool's blocks; this pool is private")
    base, capacity = pool.arena()
    out = []
    for allocation in allocations:
        if allocation.pool is not pool:
            raise ValueError("allocation belongs to another pool")
        offset = allocation.pointer - base
        if offset < 0 or offset + allocation.size > capacity:
            raise ValueError("allocation outside the pool's arena")
        out.append({"segment": pool.shared_name, "offset": offset, "length": allocation.size})
    return out


class SharedBlock:
    """One block of another owner's shared arena, usable as a ``load_scatter`` source ``(block, 0)``."""

    foreign = True
    pool = None

    def __init__(self, view, offset, size):
        self.view, self.pointer, self.size = view, view.base + offset, size

    @property
    def closed(self):
        return self.view.closed

    def _open(self):
        self.view._usable()

    def mark(self, stream=0):
        """Record that work queued on ``stream`` reads this block; the view's close waits for it."""
        self.view._fence(stream)


class SharedBlocks:
    """Another process's shared pinned arena, mapped read-only here and registered with this GPU."""

    def __init__(self, name: str, device: int = 0, library=None):
        from .dataplane import _load
        self.lib = _load(library)
        if not hasattr(self.lib, "kvsnap_shared_open"):
            raise RuntimeError("this CUDA library has no shared pools; rebuild with python -m kvsnap_b200.build")
        base, size = C.c_void_p(), C.c_size_t()
        if self.lib.kvsnap_shared_open(name.encode(), device, C.byref(base), C.byref(size)) < 0:
            raise RuntimeError(self.lib.kvsnap_cuda_error().decode())
        self.name, self.device, self.base, self.size = name, device, base.value, size.value
        self._pid = os.getpid()
        self._lock = threading.Lock()
        self._fences = []
        self.closed = False

    def _usable(self):
        if self._pid != os.getpid():
            raise RuntimeError("shared host-tier mappings must not be inherited across fork")
        if self.closed:
            raise RuntimeError("shared host-tier mapping closed")

    def _fence(self, stream):
        import torch
        event = torch.cuda.Event()
        event.record(torch.cuda.ExternalStream(stream) if stream else torch.cuda.current_stream())
        with self._lock:
            self._fences = [e for e in self._fences if not e.query()] + [event]

    def block(self, offset: int, length: int) -> SharedBlock:
        self._usable()
        if type(offset) is not int or type(length) is not int or offset < 0 or length <= 0 or \
                offset + length > self.size:
            raise ValueError("shared block outside the mapped arena")
        return SharedBlock(self, offset, length)

    def sources(self, located):
        """``load_scatter`` sources for locations from ``locations()`` that name this segment."""
        out = []
        for location in located:
            if location.get("segment") != self.name:
                raise ValueError("location names another shared segment")
            out.append((self.block(location["offset"], location["length"]), 0))
        return out

    def close(self):
        """Wait for the kernels that read the mapping, then unregister and unmap it (idempotent)."""
        if self._pid != os.getpid() or self.closed:
            return
        with self._lock:
            fences, self._fences = self._fences, []
        for event in fences:
            event.synchronize()
        if self.lib.kvsnap_shared_close(C.c_void_p(self.base), self.size) < 0:
            raise RuntimeError(self.lib.kvsnap_cuda_error().decode())
        self.closed = True

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()
