"""ORACLE harness: the reference's own data plane run on the CPU. Test infrastructure only.

The reference's ``TorchBlockDataPlane`` (kvsnap/connector/dataplane.py:214-437)
is written for CUDA tensors, its pinned pool and its Triton restore kernel.
These stand-ins let its unmodified Python run on CPU tensors: CUDA calls are
no-ops, the pinned pool is host buffers whose copies are memmoves, and the
restore kernel is a memmove per (block, layer) job over the tables the data
plane builds (the Triton kernel's semantics, kvsnap/connector/copy_kernel.py:23-40).
``tests/golden/make_golden.py`` records golden vectors through it, and the
benchmark's reference arm times the reference's CPU path through it. Nothing
in the product (``kvsnap_b200``) imports this module.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import sys
from types import SimpleNamespace
from unittest.mock import patch

import torch

class _Event:
    def record(self, stream=None):
        pass

    def synchronize(self):
        pass

    def query(self):
        return True


class _Stream:
    def synchronize(self):
        pass


class _Pinnable:
    """What ``torch.tensor`` returns here: ``pin_memory()`` is the tensor itself."""
    def __init__(self, tensor):
        self._tensor = tensor

    def pin_memory(self):
        return self._tensor

    def __getattr__(self, name):
        return getattr(self._tensor, name)


class _Torch:
    """The ``torch`` module as the reference data plane sees it, minus CUDA."""
    cuda = SimpleNamespace(stream=lambda stream: contextlib.nullcontext(), Event=_Event,
                           ExternalStream=lambda handle, device=None: _Stream())

    def __getattr__(self, name):
        return getattr(torch, name)

    def tensor(self, *args, **kwargs):
        return _Pinnable(torch.tensor(*args, **kwargs))


class _OnCuda:
    """A CPU tensor that claims a CUDA device, for the registration-time device check."""
    device = SimpleNamespace(type="cuda", index=0)

    def __init__(self, tensor):
        self._tensor = tensor

    def __getattr__(self, name):
        return getattr(self._tensor, name)

    def __getitem__(self, index):
        return self._tensor[index]


class HostBuffer:
    """A pinned allocation stand-in: a host buffer whose copies are memmoves."""
    def __init__(self, size):
        self.size, self.closed = size, False
        self._buffer = C.create_string_buffer(max(size, 1))
        self.pointer = C.addressof(self._buffer)

    def _open(self):
        if self.closed:
            raise RuntimeError("pinned allocation closed")

    def copy(self, device_ptr, size, offset=0, *, to_host, producer_stream=0):
        if offset < 0 or offset + size > self.size:
            raise ValueError("copy outside allocation")
        host = self.pointer + offset
        C.memmove(host if to_host else device_ptr, device_ptr if to_host else host, size)

    def wait(self):
        pass

    def zero(self, offset, size):
        C.memset(self.pointer + offset, 0, size)

    def read_range(self, offset, size):
        return C.string_at(self.pointer + offset, size)


class _Pool:
    @contextlib.contextmanager
    def borrow_copy_stream(self):
        yield 1

    @contextlib.contextmanager
    def operation(self):
        yield


def restore_by_memmove(sources, blocks, layer_offsets, layer_bases, layer_pitches, layer_words):
    layers = list(zip(*(t.tolist() for t in (layer_offsets, layer_bases, layer_pitches, layer_words))))
    for source, block in zip(sources.tolist(), blocks.tolist()):
        for offset, base, pitch, words in layers:
            C.memmove(base + block * pitch, source + offset, words * 8)


def register(dataplane, caches, block_size):
    with patch.dict(sys.modules, {"torch": _Torch()}), \
         patch.object(dataplane, "CudaPool", return_value=_Pool()):
        plane = dataplane.TorchBlockDataPlane({k: _OnCuda(v) for k, v in caches.items()}, block_size, 1 << 30)
    plane.caches = dict(sorted(caches.items()))
    return plane
