"""The host I/O library (kvsnap_b200/csrc/io.cpp): CRC32C values and the pread/pwrite failure rules.

CRC32C must equal the reference's (csrc/dataplane/io.cpp) on its known vectors
and every golden vector; the three-stream SSE4.2 path is checked against the
oracle over lengths and priors that cross its 24 KiB rounds. The file I/O
paths are linked against a syscall fault shim (tests/native/io_faults.c) and
must keep the reference's errno contract (tests/unit/test_native_io.py there).
"""
import ctypes as C
import errno
import os
import shutil
import subprocess
import tempfile
import threading
import time
from pathlib import Path

import pytest

import kvgen
from cases import GOLDEN
from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]
PWRITE, PREAD, FDATASYNC = 0, 1, 2
FAIL, SHORT, NOTHING = 1, 2, 3


@pytest.fixture(scope="module")
def io():
    from kvsnap_b200 import build
    from kvsnap_b200 import _abi
    return _abi.load(build.build_io(), _abi.IO_API)


@pytest.fixture(scope="module")
def faulty(tmp_path_factory):
    if not shutil.which("g++") or not shutil.which("gcc"):
        pytest.skip("compilers unavailable")
    out = tmp_path_factory.mktemp("iofaults")
    shim = out / "io_faults.o"
    subprocess.run(["gcc", "-c", "-fPIC", "-O1", str(ROOT / "tests/native/io_faults.c"), "-o", str(shim)], check=True)
    lib = out / "libiofaults.so"
    result = subprocess.run(["g++", "-std=c++17", "-shared", "-fPIC", "-pthread", "-O2", f"-I{ROOT / 'include'}",
                             str(ROOT / "kvsnap_b200/csrc/io.cpp"), str(shim), "-o", str(lib),
                             "-Wl,--wrap=pwrite,--wrap=pread,--wrap=fdatasync"], capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    from kvsnap_b200 import _abi
    handle = _abi.declare(C.CDLL(str(lib)), _abi.IO_API)
    handle.io_fault.argtypes, handle.io_fault.restype = [C.c_int] * 4, None
    handle.io_calls.argtypes, handle.io_calls.restype = [C.c_int], C.c_int
    handle.io_stall.argtypes, handle.io_stall.restype = [C.c_int], None
    handle.io_inside.restype = handle.io_peak.restype = C.c_int
    return handle


@pytest.fixture
def tmpfile():
    f = tempfile.TemporaryFile()
    yield f
    f.close()


def test_abi_version(io):
    assert io.kvsnap_io_abi_version() == 1


def test_reference_known_vectors(io):
    for value, checksum in [(b"", 0), (b"123456789", 0xE3069283), (bytes(32), 0x8A9136AA),
                            (b"\xff" * 32, 0x62A8AB43)]:
        assert io.kvsnap_crc32c(value, len(value)) == checksum


@pytest.mark.parametrize("row", GOLDEN["crc32c"], ids=lambda r: r["label"])
def test_golden_vectors(io, row):
    data = bytes.fromhex(row["hex"]) if "hex" in row else kvgen.random_bytes(row["seed"], row["length"]).tobytes()
    assert io.kvsnap_crc32c(data, len(data)) == row["crc"]
    if "split" in row:
        s = row["split"]
        first = io.kvsnap_crc32c_extend(data[:s], s, 0)
        assert io.kvsnap_crc32c_extend(data[s:], len(data) - s, first) == row["crc_extend"]
        assert io.kvsnap_crc32c_extend(data, len(data), 0x1234ABCD) == row["crc_prior_1234"]


@pytest.mark.parametrize("length", [0, 1, 7, 8, 9, 24575, 24576, 24577, 49152 + 13, 100_000, (1 << 20) + 3])
def test_interleaved_sse_path_matches_oracle(io, length):
    data = kvgen.random_bytes(length + 3, length + 5).tobytes()
    for offset in (0, 3):                  # misaligned starts too
        chunk = data[offset:offset + length]
        for prior in (0, 0xDEADBEEF):
            assert io.kvsnap_crc32c_extend(chunk, len(chunk), prior) == oracle.crc32c(chunk, prior)


def test_incremental_crc_matches_bitwise_oracle_for_unaligned_lengths(io):
    data = bytes(range(256)) * 4
    for length in (0, 1, 7, 8, 9, 15, 31, 127, 1024):
        value = data[:length]
        for split in (0, length // 2, length):
            first = io.kvsnap_crc32c_extend(value[:split], split, 0)
            assert io.kvsnap_crc32c_extend(value[split:], length - split, first) == oracle.crc32c_bitwise(value)


def test_pwrite_retries_interrupts_and_short_writes(faulty, tmpfile):
    fd = tmpfile.fileno()
    faulty.io_calls(PWRITE)
    faulty.io_fault(PWRITE, FAIL, 2, errno.EINTR)
    assert faulty.kvsnap_pwrite_all(fd, b"kv-bytes", 8, 3, 0) == 0
    assert os.pread(fd, 8, 3) == b"kv-bytes"
    assert faulty.io_calls(PWRITE) == 3
    faulty.io_fault(PWRITE, SHORT, 3, 0)
    assert faulty.kvsnap_pwrite_all(fd, b"abcdef", 6, 0, 0) == 0
    assert os.pread(fd, 6, 0) == b"abcdef"
    assert faulty.io_calls(PWRITE) == 4          # three one-byte writes, then the rest


def test_pwrite_errors_are_returned_not_hidden(faulty, tmpfile):
    fd = tmpfile.fileno()
    faulty.io_fault(PWRITE, NOTHING, 1, 0)
    assert faulty.kvsnap_pwrite_all(fd, b"x", 1, 0, 0) == errno.EIO
    faulty.io_fault(PWRITE, FAIL, 1, errno.ENOSPC)
    assert faulty.kvsnap_pwrite_all(fd, b"x", 1, 0, 0) == errno.ENOSPC
    assert faulty.kvsnap_pwrite_all(-1, b"x", 1, 0, 0) == errno.EBADF
    assert faulty.kvsnap_pwrite_all(fd, b"x", 1, -1, 0) == errno.EINVAL
    assert faulty.kvsnap_pwrite_all(fd, b"xx", 2, 2**63 - 2, 0) == errno.EINVAL
    faulty.io_fault(-1, 0, 0, 0)


def test_durable_writes_sync_and_retry_interrupted_syncs(faulty, tmpfile):
    fd = tmpfile.fileno()
    faulty.io_calls(FDATASYNC)
    assert faulty.kvsnap_pwrite_all(fd, b"", 0, 0, 1) == 0
    assert faulty.io_calls(FDATASYNC) == 1
    assert faulty.kvsnap_pwrite_all(fd, b"y", 1, 0, 0) == 0
    assert faulty.io_calls(FDATASYNC) == 0
    faulty.io_fault(FDATASYNC, FAIL, 1, errno.EINTR)
    assert faulty.kvsnap_pwrite_all(fd, b"y", 1, 0, 1) == 0
    assert faulty.io_calls(FDATASYNC) == 2
    faulty.io_fault(FDATASYNC, FAIL, 1, errno.EIO)
    assert faulty.kvsnap_pwrite_all(fd, b"y", 1, 0, 1) == errno.EIO


def test_pread_completes_short_reads_and_reports_eof(faulty, tmpfile):
    fd = tmpfile.fileno()
    payload = b"read-exact-native-bytes"
    os.pwrite(fd, payload, 0)
    out = C.create_string_buffer(len(payload))
    faulty.io_fault(PREAD, SHORT, 2, 0)
    assert faulty.kvsnap_pread_all(fd, out, len(payload), 0) == 0 and out.raw == payload
    faulty.io_fault(PREAD, FAIL, 1, errno.EINTR)
    assert faulty.kvsnap_pread_all(fd, out, len(payload), 0) == 0
    assert faulty.kvsnap_pread_all(fd, out, len(payload), 1) == errno.EIO          # one byte short at EOF
    faulty.io_fault(PREAD, NOTHING, 1, 0)
    assert faulty.kvsnap_pread_all(fd, out, 4, 0) == errno.EIO
    assert faulty.kvsnap_pread_all(fd, out, 4, -5) == errno.EINVAL


def test_worker_pool_arguments_budget_and_concurrency(io, tmpfile):
    assert not io.kvsnap_io_pool_create(0, 10) and not io.kvsnap_io_pool_create(65, 10)
    assert not io.kvsnap_io_pool_create(2, 0)
    pool = io.kvsnap_io_pool_create(4, 1 << 16)
    try:
        fd = tmpfile.fileno()
        buf = C.create_string_buffer(16)
        assert io.kvsnap_io_pool_transfer(pool, fd, buf, 16, 0, 2, 0) == errno.EINVAL
        assert io.kvsnap_io_pool_transfer(None, fd, buf, 16, 0, 1, 0) == errno.EINVAL
        assert io.kvsnap_io_pool_transfer(pool, fd, None, 16, 0, 1, 0) == errno.EINVAL
        big = C.create_string_buffer((1 << 16) + 1)
        assert io.kvsnap_io_pool_transfer(pool, fd, big, (1 << 16) + 1, 0, 1, 0) == errno.EMSGSIZE
        blocks = [kvgen.random_bytes(i, 1 << 14).tobytes() for i in range(16)]
        results = [None] * 16

        def write(i):
            results[i] = io.kvsnap_io_pool_transfer(pool, fd, blocks[i], len(blocks[i]), i << 14, 1, 0)

        threads = [threading.Thread(target=write, args=(i,)) for i in range(16)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        assert results == [0] * 16
        back = C.create_string_buffer(1 << 18)
        assert io.kvsnap_io_pool_transfer(pool, fd, back, 1 << 16, 0, 0, 0) == 0
        assert back.raw[:1 << 16] == b"".join(blocks[:4])
    finally:
        io.kvsnap_io_pool_destroy(pool)


def _until(predicate, seconds=5.0):
    deadline = time.monotonic() + seconds
    while not predicate():
        if time.monotonic() > deadline:
            return False
        time.sleep(0.01)
    return True


@pytest.mark.parametrize("slots, budget, expect", [(2, 1 << 20, 2), (8, 3 * 4096, 3)])
def test_transfer_pool_runs_at_most_its_slots_and_bytes_at_once(faulty, tmpfile, slots, budget, expect):
    """kvsnap_io_pool_create's limits: `workers` transfers and `max_bytes` in flight (reference io.cpp:130-154)."""
    pool = faulty.kvsnap_io_pool_create(slots, budget)
    fd = tmpfile.fileno()
    blocks = [kvgen.random_bytes(40 + i, 4096).tobytes() for i in range(6)]
    results = [None] * 6

    def write(i):
        results[i] = faulty.kvsnap_io_pool_transfer(pool, fd, blocks[i], 4096, i * 4096, 1, 0)

    faulty.io_peak()
    faulty.io_stall(1)
    threads = [threading.Thread(target=write, args=(i,)) for i in range(6)]
    try:
        for t in threads:
            t.start()
        assert _until(lambda: faulty.io_inside() == expect)
        time.sleep(0.2)
        assert faulty.io_inside() == expect          # the rest wait for a slot or for bytes
    finally:
        faulty.io_stall(0)
        for t in threads:
            t.join(10)
    assert results == [0] * 6 and faulty.io_peak() == expect
    back = C.create_string_buffer(6 * 4096)
    assert faulty.kvsnap_pread_all(fd, back, 6 * 4096, 0) == 0
    assert back.raw == b"".join(blocks)
    faulty.kvsnap_io_pool_destroy(pool)


def test_destroying_the_transfer_pool_cancels_waiters_and_waits_for_running(faulty, tmpfile):
    pool = faulty.kvsnap_io_pool_create(1, 1 << 20)
    fd = tmpfile.fileno()
    data = kvgen.random_bytes(7, 4096).tobytes()
    results = {}

    def write(key):
        results[key] = faulty.kvsnap_io_pool_transfer(pool, fd, data, 4096, 0, 1, 0)

    faulty.io_stall(1)
    running = threading.Thread(target=write, args=("running",))
    waiting = threading.Thread(target=write, args=("waiting",))
    destroy = threading.Thread(target=faulty.kvsnap_io_pool_destroy, args=(pool,))
    try:
        running.start()
        assert _until(lambda: faulty.io_inside() == 1)
        waiting.start()
        time.sleep(0.1)
        destroy.start()
        assert _until(lambda: "waiting" in results)
        assert results["waiting"] == errno.ECANCELED
        time.sleep(0.1)
        assert destroy.is_alive() and "running" not in results     # the admitted transfer holds the pool
    finally:
        faulty.io_stall(0)
        for t in (running, waiting, destroy):
            t.join(10)
    assert results["running"] == 0 and not destroy.is_alive()


def test_native_io_wrapper_round_trip(tmpfile):
    from kvsnap_b200.native_io import get_io_backend
    from kvsnap_b200.crc32c import crc32c
    backend = get_io_backend()
    assert backend is get_io_backend("native")
    data = kvgen.random_bytes(11, 200_000).tobytes()
    fd = tmpfile.fileno()
    backend.pwrite_all(fd, data, 7)
    assert backend.pread_all(fd, len(data), 7) == data
    target = C.create_string_buffer(len(data))
    backend.pread_into(fd, C.addressof(target), len(data), 7)
    assert target.raw == data
    assert backend.crc32c_at(C.addressof(target), len(data)) == oracle.crc32c(data) == crc32c(data)
    assert crc32c(data[1000:], crc32c(data[:1000])) == crc32c(data)
    with pytest.raises(ValueError):
        crc32c(b"x", -1)
    with pytest.raises(ValueError):
        backend.pread_all(fd, -1, 0)
    with pytest.raises(OSError):
        backend.pread_all(fd, 10, 10 ** 9)
    with pytest.raises(ValueError):
        get_io_backend("python")


def test_native_io_pieces_close_and_fork_rules(tmpfile):
    """NativeIO's own contract (reference native_io.py:51-151): transfers above the byte budget go in pieces,
    a closed backend and one inherited across fork refuse work, and close is idempotent."""
    from unittest.mock import patch
    from kvsnap_b200.native_io import NativeIO, resolve_io_library
    backend = NativeIO(resolve_io_library(), workers=3, queue_bytes=4096)
    fd = tmpfile.fileno()
    data = kvgen.random_bytes(99, 3 * 4096 + 123).tobytes()
    backend.pwrite_all(fd, bytearray(data), 5)
    assert backend.pread_all(fd, len(data), 5) == data
    target = C.create_string_buffer(len(data))
    backend.pread_into(fd, C.addressof(target), len(data), 5)
    backend.pwrite_from(fd, C.addressof(target), len(data), 5 + len(data))
    assert backend.pread_all(fd, 2 * len(data), 5) == data + data
    assert backend.crc32c(memoryview(data)) == oracle.crc32c(data)
    for bad in ((-1, 0), (1, -1), (2**62, 2**62), (1.0, 0)):
        with pytest.raises(ValueError, match="invalid I/O range"):
            backend.pread_all(fd, *bad)
    with pytest.raises(ValueError, match="capacity"):
        NativeIO(resolve_io_library(), workers=0)
    with patch("os.getpid", return_value=os.getpid() + 1):
        with pytest.raises(RuntimeError, match="fork"):
            backend.pread_all(fd, 4, 0)
        backend.close()                       # a child leaves the parent's pool alone
    assert backend.handle
    backend.close()
    backend.close()
    with pytest.raises(RuntimeError, match="closed"):
        backend.pread_all(fd, 4, 0)
    with pytest.raises(RuntimeError, match="closed"):
        backend.crc32c(b"x")
