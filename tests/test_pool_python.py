"""CudaPool / PinnedAllocation (kvsnap_b200/dataplane.py) over the real pool C++ built against the fake runtime.

The Python owners carry the reference's lifetime rules (kvsnap/connector/dataplane.py:38-211,
tested there by tests/connector/test_native_lifetime.py): reservations map
"pinned capacity exhausted" to PinnedCapacityError, every entry refuses a
closed pool or a forked process, a close waits for an operation in progress,
and a failed close keeps the pool and its allocations alive.
"""
import ctypes as C
import os
import shutil
import subprocess
import threading
import time
from pathlib import Path
from unittest.mock import patch

import pytest

ROOT = Path(__file__).resolve().parents[1]
NATIVE = ROOT / "tests" / "native"


@pytest.fixture(scope="module")
def fake_library(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ unavailable")
    out = tmp_path_factory.mktemp("fakepool") / "libfakepool_py.so"
    cmd = ["g++", "-std=c++17", "-shared", "-fPIC", "-Wl,-Bsymbolic", "-I", str(NATIVE),
           "-I", str(ROOT / "kvsnap_b200" / "csrc"), "-I", str(ROOT / "include"),
           str(ROOT / "kvsnap_b200" / "csrc" / "pool.cpp"), str(NATIVE / "fake_cudart.cpp"), "-o", str(out)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    lib = C.CDLL(str(out))
    lib.fake_cuda_fail_next.argtypes = [C.c_char_p]
    lib.fake_cuda_pending.restype = C.c_int
    return out, lib


@pytest.fixture
def pool(fake_library):
    from kvsnap_b200.dataplane import CudaPool
    path, _ = fake_library
    p = CudaPool(1024, 0, library=str(path))
    yield p
    if p.handle:
        p.close()


def test_reserve_maps_capacity_errors(pool):
    from kvsnap_b200.dataplane import PinnedCapacityError
    a = pool.reserve(512)
    assert a.size == 512 and a.pointer
    with pytest.raises(PinnedCapacityError):
        pool.reserve(1024)
    a.close()
    assert pool.reserve(1024).size == 1024


def test_copy_wait_read_write_and_bounds(pool, fake_library):
    _, lib = fake_library
    a = pool.reserve(32)
    a.write(bytes(range(32)))
    assert a.read() == bytes(range(32))
    device = C.create_string_buffer(32)
    a.copy(C.addressof(device), 32, 0, to_host=False)
    assert lib.fake_cuda_pending() == 1 and not a.ready()
    a.wait()
    assert device.raw == bytes(range(32)) and a.ready()
    with pytest.raises(RuntimeError, match="outside"):
        a.copy(C.addressof(device), 33, 0, to_host=False)
    with pytest.raises(ValueError):
        a.read_range(30, 4)
    with pytest.raises(ValueError):
        a.copy(-1, 4, 0, to_host=True)
    a.zero(0, 8)
    assert a.read_range(0, 8) == bytes(8)
    with pytest.raises(ValueError):
        a.write(b"short")


def test_closed_pool_and_allocations_refuse_work(pool):
    a = pool.reserve(64)
    pool.close()
    assert a.closed
    with pytest.raises(RuntimeError, match="closed"):
        a.read()
    with pytest.raises(RuntimeError, match="closed"):
        pool.reserve(1)
    a.close()                              # idempotent after the pool is gone
    pool.close()


def test_inherited_pool_refuses_use(pool):
    with patch("os.getpid", return_value=os.getpid() + 1):
        with pytest.raises(RuntimeError, match="fork"):
            pool.reserve(8)
        with pytest.raises(RuntimeError, match="fork"):
            pool.close()


def test_close_waits_for_an_operation_in_progress(pool):
    a = pool.reserve(64)
    entered, release = threading.Event(), threading.Event()
    order = []

    def hold():
        with a.operation():
            entered.set()
            release.wait(5)
            order.append("operation")

    worker = threading.Thread(target=hold)
    worker.start()
    entered.wait(5)
    closer = threading.Thread(target=lambda: (pool.close(), order.append("close")))
    closer.start()
    time.sleep(0.2)
    assert order == []                      # the close is blocked behind the operation
    release.set()
    worker.join(5)
    closer.join(5)
    assert order == ["operation", "close"]


def test_failed_close_keeps_the_pool_and_its_allocations(pool, fake_library):
    _, lib = fake_library
    a = pool.reserve(64)
    a._tensor_references = [object()]
    device = C.create_string_buffer(64)
    a.copy(C.addressof(device), 64, 0, to_host=False)
    lib.fake_cuda_fail_next(b"cudaStreamSynchronize")
    with pytest.raises(RuntimeError):
        pool.close()
    assert pool.handle and not a.closed and a._tensor_references      # owners survive a failed drain
    a.wait()
    pool.close()
    assert a.closed and not a._tensor_references


def test_borrowed_stream_handle(pool):
    with pool.borrow_copy_stream() as handle:
        assert handle
    assert pool.stream_handle() == handle


def test_copy_many_and_wait_many(pool, fake_library):
    _, lib = fake_library
    a, b = pool.reserve(16), pool.reserve(16)
    a.write(b"a" * 16)
    b.write(b"b" * 16)
    device = C.create_string_buffer(32)
    dev = C.addressof(device)
    pool.copy_many([(a, 0, dev, 16), (b, 4, dev + 16, 12)], to_host=False)
    assert lib.fake_cuda_pending() == 2 and not a.ready()
    pool.wait_many([a, b])
    assert device.raw[:28] == b"a" * 16 + b"b" * 12
    pool.copy_many([], to_host=True)
    with pytest.raises(RuntimeError, match="outside"):
        pool.copy_many([(a, 0, dev, 16), (b, 8, dev, 16)], to_host=True)
    assert lib.fake_cuda_pending() == 0
    with pytest.raises(ValueError):
        pool.copy_many([(a, -1, dev, 4)], to_host=True)
    a.close()
    with pytest.raises(RuntimeError, match="closed"):
        pool.copy_many([(a, 0, dev, 4)], to_host=True)
    with pytest.raises(RuntimeError, match="closed"):
        pool.wait_many([a])
