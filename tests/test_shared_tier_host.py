"""The cross-owner host tier on the CPU: a shared pinned pool mapped by another process.

kvsnap_b200/csrc/pool.cpp built against the fake CUDA runtime. The owner's pool
is POSIX shared memory; a second process maps it by name through
kvsnap_b200.sharedtier and reads the owner's blocks in place, the bytes the
reference's socket fetch would copy (kvsnap/connector/volatile.py:124-138).
Also: the segment is private to the user (mode 0600), the name goes with the
owner's pool while a mapping made before stays readable, names are checked,
and a name in use is refused.
"""
import ctypes as C
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
NATIVE = ROOT / "tests" / "native"

CONSUMER = r"""
import ctypes as C, hashlib, json, sys
sys.path.insert(0, sys.argv[1])
from kvsnap_b200.sharedtier import SharedBlocks
name, library, located = sys.argv[2], sys.argv[3], json.loads(sys.argv[4])
view = SharedBlocks(name, 0, library=library)
print("mapped", flush=True)
sys.stdin.readline()                      # the owner may close its pool meanwhile
sources = view.sources(located)
print(json.dumps([hashlib.sha256(C.string_at(b.pointer, b.size)).hexdigest() for b, _ in sources]), flush=True)
view.close()
"""


@pytest.fixture(scope="module")
def fake_pool_library(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ unavailable")
    out = tmp_path_factory.mktemp("sharedtier") / "libkvsnap_pool_fake.so"
    result = subprocess.run(["g++", "-std=c++17", "-shared", "-fPIC", "-Wl,-Bsymbolic", "-I", str(NATIVE),
                             "-I", str(ROOT / "kvsnap_b200" / "csrc"), "-I", str(ROOT / "include"),
                             str(ROOT / "kvsnap_b200" / "csrc" / "pool.cpp"), str(NATIVE / "fake_cudart.cpp"),
                             "-o", str(out)], capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    lib = C.CDLL(str(out))
    lib.fake_cuda_live_host_registrations.restype = C.c_int
    return out, lib


def test_another_process_reads_the_owners_blocks_in_place(fake_pool_library):
    import hashlib
    from kvsnap_b200.dataplane import CudaPool
    from kvsnap_b200.sharedtier import locations, new_segment_name
    path, fake = fake_pool_library
    name = new_segment_name()
    registered = fake.fake_cuda_live_host_registrations()
    pool = CudaPool(1 << 20, 0, library=str(path), shared_name=name)
    try:
        assert fake.fake_cuda_live_host_registrations() == registered + 1
        assert (os.stat("/dev/shm" + name).st_mode & 0o777) == 0o600
        blocks = [os.urandom(4096 * k + 48) for k in (1, 2, 3)]
        owned = [pool.reserve(len(b)) for b in blocks]
        for allocation, data in zip(owned, blocks):
            allocation.write(data)
        located = locations(pool, owned)
        assert [loc["length"] for loc in located] == [len(b) for b in blocks]
        consumer = subprocess.Popen([sys.executable, "-c", CONSUMER, str(ROOT), name, str(path), json.dumps(located)],
                                    stdin=subprocess.PIPE, stdout=subprocess.PIPE, text=True)
        try:
            assert consumer.stdout.readline().strip() == "mapped"
            for allocation in owned:
                allocation.close()
            pool.close()                                  # the name goes; the consumer's mapping stays
            assert not os.path.exists("/dev/shm" + name)
            consumer.stdin.write("go\n")
            consumer.stdin.flush()
            digests = json.loads(consumer.stdout.readline())
            assert consumer.wait(30) == 0
        finally:
            if consumer.poll() is None:
                consumer.kill()
        assert digests == [hashlib.sha256(b).hexdigest() for b in blocks]
        assert fake.fake_cuda_live_host_registrations() == registered
    finally:
        if pool.handle:
            pool.close()


def test_shared_names_are_checked_and_never_reused(fake_pool_library):
    from kvsnap_b200.dataplane import CudaPool
    from kvsnap_b200.sharedtier import SharedBlocks, new_segment_name
    path, _ = fake_pool_library
    for bad in ("no-slash", "/two/parts", "/"):
        with pytest.raises(RuntimeError, match="one path component"):
            CudaPool(4096, 0, library=str(path), shared_name=bad)
    name = new_segment_name()
    pool = CudaPool(4096, 0, library=str(path), shared_name=name)
    try:
        with pytest.raises(RuntimeError, match="shm_open"):
            CudaPool(4096, 0, library=str(path), shared_name=name)      # a name in use is refused
        view = SharedBlocks(name, 0, library=str(path))
        with pytest.raises(ValueError, match="outside"):
            view.block(4000, 200)
        with pytest.raises(ValueError, match="another shared segment"):
            view.sources([{"segment": "/kvsnap-other", "offset": 0, "length": 16}])
        view.close()
        with pytest.raises(RuntimeError, match="closed"):
            view.block(0, 16)
    finally:
        pool.close()
    with pytest.raises(RuntimeError, match="shm_open"):
        SharedBlocks(name, 0, library=str(path))                          # gone with its pool
