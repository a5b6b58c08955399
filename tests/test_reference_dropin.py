"""The reference's own Python pool classes over this repository's pool library, on the CPU.

kvsnap's connector binds the pinned pool through its own
``kvsnap.connector.dataplane.CudaPool`` / ``PinnedAllocation`` (reference
dataplane.py:38-211), resolving the C library through ``KVSNAP_CUDA_LIBRARY``.
Here those classes, imported from the installed reference, drive
``kvsnap_b200/csrc/pool.cpp`` built against a fake CUDA runtime: the ABI
version check, reservations and the "pinned capacity exhausted" mapping,
copies in both directions and their bounds errors, strided copies, wait and
ready, host reads and writes, the borrowed copy stream, and a close whose
drain fails keeping the pool and its allocations. The reference's own tests of
the same rules mock its ABI in Python (tests/connector/test_native_lifetime.py)
or build its own pool (tests/unit/test_independent_native.py); these run its
classes on our library instead.
"""
import ctypes as C
import shutil
import subprocess
from pathlib import Path

import pytest

from refpath import reference

ROOT = Path(__file__).resolve().parents[1]
NATIVE = ROOT / "tests" / "native"


@pytest.fixture(scope="module")
def our_pool_library(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ unavailable")
    out = tmp_path_factory.mktemp("dropin") / "libkvsnap_pool_fake.so"
    result = subprocess.run(["g++", "-std=c++17", "-shared", "-fPIC", "-Wl,-Bsymbolic", "-I", str(NATIVE),
                             "-I", str(ROOT / "kvsnap_b200" / "csrc"), "-I", str(ROOT / "include"),
                             str(ROOT / "kvsnap_b200" / "csrc" / "pool.cpp"), str(NATIVE / "fake_cudart.cpp"),
                             "-o", str(out)], capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    fake = C.CDLL(str(out))
    fake.fake_cuda_fail_next.argtypes = [C.c_char_p]
    fake.fake_cuda_pending.restype = C.c_int
    return out, fake


@pytest.fixture
def ref_pool(our_pool_library, monkeypatch):
    dataplane = reference("connector.dataplane")
    path, fake = our_pool_library
    monkeypatch.setenv("KVSNAP_CUDA_LIBRARY", str(path))
    assert dataplane.resolve_cuda_library() == path
    pool = dataplane.CudaPool(4096, 0)
    yield dataplane, pool, fake
    if pool.handle:
        pool.close()


def test_reference_pool_class_runs_on_our_library(ref_pool):
    dataplane, pool, fake = ref_pool
    assert pool.abi_version == 2
    a = pool.reserve(1024)
    assert isinstance(a, dataplane.PinnedAllocation) and a.size == 1024 and a.pointer % 16 == 0
    with pytest.raises(dataplane.PinnedCapacityError, match="pinned capacity exhausted"):
        pool.reserve(4096)
    a.write(bytes(range(256)) * 4)
    device = C.create_string_buffer(1024)
    a.copy(C.addressof(device), 1024, to_host=False)
    assert fake.fake_cuda_pending() == 1 and not a.ready()
    a.wait()
    assert a.ready() and device.raw == bytes(range(256)) * 4
    a.zero(0, 256)
    a.copy(C.addressof(device), 256, 768, to_host=True)          # device bytes 0..255 -> host 768..1023
    assert a.read_range(768, 256) == bytes(range(256))
    assert a.read_range(0, 256) == bytes(256)
    with pytest.raises(RuntimeError, match="outside"):
        a.copy(C.addressof(device), 1025, to_host=True)
    with pytest.raises(ValueError):
        a.copy(C.addressof(device), -1, to_host=True)
    # Strided: bytes 4..7 of each of 3 rows of 8 on the host, rows of 6 on the device.
    b = pool.reserve(24)
    b.write(bytes(range(24)))
    strided = C.create_string_buffer(b"\xee" * 18, 18)
    b.copy_2d(C.addressof(strided), 6, 4, 8, 4, 3, to_host=False)
    b.wait()
    assert strided.raw == bytes([4, 5, 6, 7, 0xEE, 0xEE, 12, 13, 14, 15, 0xEE, 0xEE, 20, 21, 22, 23, 0xEE, 0xEE])
    with pytest.raises(RuntimeError, match="outside"):
        b.copy_2d(C.addressof(strided), 6, 4, 8, 5, 3, to_host=False)
    with pool.borrow_copy_stream() as handle:
        assert handle
    a.close()
    b.close()
    assert pool.reserve(4096).size == 4096


def test_reference_pool_class_keeps_everything_when_the_drain_fails(ref_pool):
    dataplane, pool, fake = ref_pool
    a = pool.reserve(64)
    a._tensor_references = [object()]
    device = C.create_string_buffer(64)
    a.copy(C.addressof(device), 64, to_host=False)
    fake.fake_cuda_fail_next(b"cudaStreamSynchronize")
    with pytest.raises(RuntimeError):
        pool.close()
    assert pool.handle and not a.closed and a._tensor_references
    pool.close()
    assert a.closed and not a._tensor_references
    with pytest.raises(RuntimeError, match="closed"):
        pool.reserve(8)
