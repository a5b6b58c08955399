"""The pinned pool's C++ control path (kvsnap_b200/csrc/pool.cpp) against a fake CUDA runtime, on a CPU.

The fake (tests/native/fake_cudart.*) queues copies and applies them only at a
synchronize, and can fail any call once, so these tests reach the failure rules
of the reference's pool ABI 2 (kvsnap csrc/dataplane/cuda_pool.cpp, tested by
its tests/unit/test_independent_native.py and test_native_lifetime.py):
an allocation is never released while a copy may still touch it, a failed
drain keeps the memory, geometry and capacity are checked before any copy.
They prove control flow only, never CUDA behaviour.
"""
import ctypes as C
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
NATIVE = ROOT / "tests" / "native"


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ unavailable")
    out = tmp_path_factory.mktemp("fakepool") / "libfakepool.so"
    # -Bsymbolic binds the pool to this fake even when a real CUDA runtime is loaded in the process.
    cmd = ["g++", "-std=c++17", "-shared", "-fPIC", "-Wl,-Bsymbolic", "-Wall", "-Wextra", "-Werror",
           "-I", str(NATIVE), "-I", str(ROOT / "kvsnap_b200" / "csrc"), "-I", str(ROOT / "include"),
           str(ROOT / "kvsnap_b200" / "csrc" / "pool.cpp"), str(NATIVE / "fake_cudart.cpp"), "-o", str(out)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    assert result.returncode == 0, result.stderr
    lib = C.CDLL(str(out))
    from kvsnap_b200 import _abi
    _abi.declare(lib, _abi.POOL_API)
    _abi.declare(lib, _abi.POOL_EXTRA)
    lib.fake_cuda_fail_next.argtypes, lib.fake_cuda_fail_next.restype = [C.c_char_p], None
    lib.fake_cuda_pending.restype = C.c_int
    lib.fake_cuda_live_host_allocations.restype = C.c_int
    lib.fake_cuda_last_stream.restype = C.c_size_t
    return lib


def reserve(lib, pool, size):
    ident, ptr = C.c_uint64(), C.c_void_p()
    rc = lib.kvsnap_pool_reserve(pool, size, C.byref(ident), C.byref(ptr))
    return rc, ident.value, ptr.value


def error(lib):
    return lib.kvsnap_cuda_error().decode()


def test_abi_version_and_create_failures(lib):
    assert lib.kvsnap_pool_abi_version() == 2
    assert not lib.kvsnap_pool_create(0, 0)
    assert "positive" in error(lib)
    lib.fake_cuda_fail_next(b"cudaHostAlloc")
    assert not lib.kvsnap_pool_create(64, 0)
    assert error(lib) == "injected CUDA error"


def test_reservations_are_first_fit_16_byte_aligned_and_capacity_checked(lib):
    pool = lib.kvsnap_pool_create(256, 0)
    try:
        rc, a, pa = reserve(lib, pool, 40)
        rc2, b, pb = reserve(lib, pool, 64)
        assert rc == rc2 == 0 and pb - pa == 48          # 40 rounded up to 48
        rc, _, _ = reserve(lib, pool, 1024)
        assert rc == -1 and "pinned capacity exhausted" in error(lib)
        rc, _, _ = reserve(lib, pool, 0)
        assert rc == -1 and "pinned capacity exhausted" in error(lib)
        assert lib.kvsnap_pool_release(pool, a) == 0
        rc, c, pc = reserve(lib, pool, 32)                # reuses the hole before b
        assert rc == 0 and pc == pa
        rc, _, _ = reserve(lib, pool, 256 - 112 + 1)      # 112 = end of b; one byte too many
        assert rc == -1
        assert lib.kvsnap_pool_release(pool, 999) == -1 and "unknown pinned allocation" in error(lib)
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_copies_stay_queued_until_waited_and_release_drains_them(lib):
    pool = lib.kvsnap_pool_create(64, 0)
    try:
        rc, a, ptr = reserve(lib, pool, 16)
        C.memmove(ptr, b"0123456789abcdef", 16)
        device = C.create_string_buffer(16)
        assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 16, 0, 0) == 0
        assert lib.fake_cuda_pending() == 1 and device.raw == bytes(16)
        assert lib.kvsnap_pool_ready(pool, a) == 0
        assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 17, 0, 0) == -1
        assert "outside pinned allocation" in error(lib)
        assert lib.kvsnap_pool_wait(pool, a) == 0
        assert device.raw == b"0123456789abcdef" and lib.kvsnap_pool_ready(pool, a) == 1
        stream = C.c_size_t()
        assert lib.kvsnap_pool_copy_stream(pool, C.byref(stream)) == 0
        assert stream.value == lib.fake_cuda_last_stream()
        assert lib.kvsnap_pool_copy(pool, a, 8, C.addressof(device), 8, 1, 0) == 0    # D2H into the slot
        assert lib.kvsnap_pool_release(pool, a) == 0                                  # blocking release
        assert lib.fake_cuda_pending() == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_failed_event_record_never_frees_inflight_bytes(lib):
    pool = lib.kvsnap_pool_create(32, 0)
    try:
        rc, a, _ = reserve(lib, pool, 32)
        device = C.create_string_buffer(32)
        lib.fake_cuda_fail_next(b"cudaEventRecord")
        assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 32, 0, 0) == -1
        assert lib.fake_cuda_pending() == 1            # the copy itself was queued
        # The stale event cannot vouch for the copy: release drains the stream.
        assert lib.kvsnap_pool_release(pool, a) == 0
        assert lib.fake_cuda_pending() == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_failed_drain_keeps_the_allocation_out_of_reuse(lib):
    pool = lib.kvsnap_pool_create(16, 0)
    try:
        rc, a, _ = reserve(lib, pool, 16)
        device = C.create_string_buffer(16)
        lib.fake_cuda_fail_next(b"cudaEventRecord")
        assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 16, 0, 0) == -1
        lib.fake_cuda_fail_next(b"cudaStreamSynchronize")
        assert lib.kvsnap_pool_release(pool, a) == -1
        assert lib.fake_cuda_pending() == 1
        assert reserve(lib, pool, 1)[0] == -1           # still owned
        assert lib.kvsnap_pool_release(pool, a) == 0    # a later drain succeeds
        assert lib.fake_cuda_pending() == 0
        assert reserve(lib, pool, 16)[0] == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_failed_enqueue_falls_back_to_draining(lib):
    pool = lib.kvsnap_pool_create(16, 0)
    try:
        rc, a, _ = reserve(lib, pool, 16)
        device = C.create_string_buffer(16)
        lib.fake_cuda_fail_next(b"cudaMemcpyAsync")
        assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 16, 0, 0) == -1
        assert lib.kvsnap_pool_ready(pool, a) == 1       # nothing queued, stream idle
        assert lib.kvsnap_pool_release(pool, a) == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_producer_fence_failure_queues_nothing(lib):
    pool = lib.kvsnap_pool_create(16, 0)
    try:
        rc, a, _ = reserve(lib, pool, 16)
        device = C.create_string_buffer(16)
        lib.fake_cuda_fail_next(b"cudaStreamWaitEvent")
        assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 16, 1, 0) == -1
        assert lib.fake_cuda_pending() == 0
        assert lib.kvsnap_pool_release(pool, a) == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_strided_copy_moves_one_layer_of_consecutive_blocks_and_checks_bounds(lib):
    # Three packed blocks of 8 bytes; layer 1 is bytes 4..7 of each. Device rows: pitch 6, first 4 bytes.
    pool = lib.kvsnap_pool_create(24, 0)
    try:
        rc, a, ptr = reserve(lib, pool, 24)
        C.memmove(ptr, bytes(range(24)), 24)
        device = C.create_string_buffer(b"\xee" * 18, 18)
        assert lib.kvsnap_pool_copy_2d(pool, a, 4, 8, C.addressof(device), 6, 4, 3, 0, 0) == 0
        assert lib.kvsnap_pool_wait(pool, a) == 0
        assert device.raw == bytes([4, 5, 6, 7, 0xee, 0xee, 12, 13, 14, 15, 0xee, 0xee, 20, 21, 22, 23, 0xee, 0xee])
        # Last row would end at 4 + 2*8 + 5 = 25 > 24.
        assert lib.kvsnap_pool_copy_2d(pool, a, 4, 8, C.addressof(device), 6, 5, 3, 0, 0) == -1
        # Pitches narrower than a row, or empty geometry.
        assert lib.kvsnap_pool_copy_2d(pool, a, 0, 2, C.addressof(device), 6, 4, 3, 0, 0) == -1
        assert lib.kvsnap_pool_copy_2d(pool, a, 0, 8, C.addressof(device), 6, 0, 3, 0, 0) == -1
        # A height whose extent overflows size_t is rejected, not wrapped.
        assert lib.kvsnap_pool_copy_2d(pool, a, 0, 1 << 62, C.addressof(device), 6, 4, 8, 0, 0) == -1
        assert lib.kvsnap_pool_release(pool, a) == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_mark_fences_in_place_work_under_the_allocation(lib):
    pool = lib.kvsnap_pool_create(32, 0)
    try:
        rc, a, _ = reserve(lib, pool, 16)
        rc, b, pb = reserve(lib, pool, 16)
        device = C.create_string_buffer(16)
        assert lib.kvsnap_pool_copy(pool, b, 0, C.addressof(device), 16, 0, 0) == 0   # other slot's copy
        assert lib.kvsnap_pool_ready(pool, a) == 1        # a has nothing queued
        assert lib.kvsnap_pool_mark(pool, a, 0) == 0      # e.g. a kernel read a in place after that copy
        assert lib.kvsnap_pool_ready(pool, a) == 0
        assert lib.kvsnap_pool_wait(pool, a) == 0
        assert lib.kvsnap_pool_ready(pool, a) == 1 and lib.fake_cuda_pending() == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_close_checked_keeps_the_pool_when_it_cannot_drain(lib):
    before = lib.fake_cuda_live_host_allocations()
    pool = lib.kvsnap_pool_create(16, 0)
    rc, a, _ = reserve(lib, pool, 16)
    device = C.create_string_buffer(16)
    assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 16, 0, 0) == 0
    lib.fake_cuda_fail_next(b"cudaStreamSynchronize")
    assert lib.kvsnap_pool_close_checked(pool) == -1
    assert lib.fake_cuda_live_host_allocations() == before + 1      # memory kept
    assert lib.kvsnap_pool_wait(pool, a) == 0                        # pool still usable
    assert lib.kvsnap_pool_close_checked(pool) == 0
    assert lib.fake_cuda_live_host_allocations() == before


def test_destroy_quarantines_memory_it_cannot_prove_idle(lib):
    before = lib.fake_cuda_live_host_allocations()
    pool = lib.kvsnap_pool_create(16, 0)
    rc, a, _ = reserve(lib, pool, 16)
    device = C.create_string_buffer(16)
    assert lib.kvsnap_pool_copy(pool, a, 0, C.addressof(device), 16, 0, 0) == 0
    lib.fake_cuda_fail_next(b"cudaStreamSynchronize")
    lib.kvsnap_pool_destroy(pool)
    assert lib.fake_cuda_live_host_allocations() == before + 1      # leaked on purpose, never reused
    assert lib.fake_cuda_pending() == 1
    lib.fake_cuda_discard_pending()      # its target buffer is about to go away


def test_mark_on_a_foreign_stream_drains_the_device_when_its_event_fails(lib):
    pool = lib.kvsnap_pool_create(32, 0)
    try:
        rc, a, _ = reserve(lib, pool, 16)
        rc, b, _ = reserve(lib, pool, 16)
        device = C.create_string_buffer(16)
        assert lib.kvsnap_pool_copy(pool, b, 0, C.addressof(device), 16, 0, 0) == 0
        lib.fake_cuda_fail_next(b"cudaEventRecord")
        assert lib.kvsnap_pool_mark(pool, a, 12345) == -1      # a kernel on another stream, unrecorded
        assert lib.kvsnap_pool_ready(pool, a) == 0              # the pool cannot vouch for it
        assert lib.kvsnap_pool_release(pool, a) == 0            # so release drains the whole device
        assert lib.fake_cuda_pending() == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_copy_on_another_stream_is_fenced_by_its_own_event(lib):
    pool = lib.kvsnap_pool_create(32, 0)
    try:
        rc, a, ptr = reserve(lib, pool, 16)
        C.memmove(ptr, b"fedcba9876543210", 16)
        device = C.create_string_buffer(16)
        assert lib.kvsnap_pool_copy_on(pool, a, 0, C.addressof(device), 16, 0, 777) == 0
        assert lib.fake_cuda_last_stream() == 777
        assert lib.kvsnap_pool_ready(pool, a) == 0
        assert lib.kvsnap_pool_copy_on(pool, a, 8, C.addressof(device), 9, 0, 777) == -1    # outside
        assert lib.kvsnap_pool_wait(pool, a) == 0
        assert device.raw == b"fedcba9876543210"
        lib.fake_cuda_fail_next(b"cudaEventRecord")
        assert lib.kvsnap_pool_copy_on(pool, a, 0, C.addressof(device), 16, 1, 777) == -1
        assert lib.kvsnap_pool_release(pool, a) == 0          # drains the device: the copy ran elsewhere
        assert lib.fake_cuda_pending() == 0
    finally:
        lib.kvsnap_pool_destroy(pool)


def _arrays(*columns):
    return [(C.c_uint64 * len(col))(*col) for col in columns]


def test_copy_many_checks_every_entry_before_queueing_any(lib):
    pool = lib.kvsnap_pool_create(64, 0)
    try:
        _, a, pa = reserve(lib, pool, 16)
        _, b, pb = reserve(lib, pool, 16)
        C.memmove(pa, b"A" * 16, 16)
        C.memmove(pb, b"B" * 16, 16)
        device = C.create_string_buffer(48)
        dev = C.addressof(device)
        # The third entry runs past its allocation: nothing at all is queued.
        ids, offs, ptrs, sizes = _arrays([a, b, b], [0, 0, 8], [dev, dev + 16, dev + 32], [16, 16, 9])
        assert lib.kvsnap_pool_copy_many(pool, 3, ids, offs, ptrs, sizes, 0, 0) == -1
        assert "outside" in error(lib) and lib.fake_cuda_pending() == 0
        ids, offs, ptrs, sizes = _arrays([a, 99], [0, 0], [dev, dev], [16, 16])
        assert lib.kvsnap_pool_copy_many(pool, 2, ids, offs, ptrs, sizes, 0, 0) == -1
        assert "unknown pinned allocation" in error(lib) and lib.fake_cuda_pending() == 0
        # A valid list: copies in order on the given stream, each allocation fenced by its event.
        ids, offs, ptrs, sizes = _arrays([a, b, b], [0, 0, 8], [dev, dev + 16, dev + 32], [16, 8, 8])
        assert lib.kvsnap_pool_copy_many(pool, 3, ids, offs, ptrs, sizes, 0, 555) == 0
        # The first two entries continue each other on both sides and move as one copy.
        assert lib.fake_cuda_last_stream() == 555 and lib.fake_cuda_pending() == 2
        assert lib.kvsnap_pool_ready(pool, a) == 0 and lib.kvsnap_pool_ready(pool, b) == 0
        waits = _arrays([a, b])[0]
        assert lib.kvsnap_pool_wait_many(pool, 2, waits) == 0
        assert device.raw[:40] == b"A" * 16 + b"B" * 8 + b"\0" * 8 + b"B" * 8
        assert lib.kvsnap_pool_copy_many(pool, 0, None, None, None, None, 0, 0) == 0
        assert lib.kvsnap_pool_copy_many(pool, -1, None, None, None, None, 0, 0) == -1
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_copy_many_failures_fall_back_to_draining(lib):
    pool = lib.kvsnap_pool_create(64, 0)
    try:
        _, a, pa = reserve(lib, pool, 16)
        _, b, pb = reserve(lib, pool, 16)
        device = C.create_string_buffer(32)
        dev = C.addressof(device)
        ids, offs, ptrs, sizes = _arrays([a, b], [0, 0], [dev, dev + 16], [16, 16])
        lib.fake_cuda_fail_next(b"cudaEventRecord")            # the first allocation's event is lost
        assert lib.kvsnap_pool_copy_many(pool, 2, ids, offs, ptrs, sizes, 1, 0) == -1
        assert lib.kvsnap_pool_release(pool, a) == 0            # no event: release drains the pool stream
        assert lib.fake_cuda_pending() == 0
        lib.fake_cuda_fail_next(b"cudaMemcpyAsync")            # the first copy is refused
        ids, offs, ptrs, sizes = _arrays([b], [0], [dev], [16])
        assert lib.kvsnap_pool_copy_many(pool, 1, ids, offs, ptrs, sizes, 1, 777) == -1
        assert lib.kvsnap_pool_ready(pool, b) in (0, 1)
        waits = _arrays([b])[0]
        assert lib.kvsnap_pool_wait_many(pool, 1, waits) == 0   # a foreign stream without an event: drain
        assert lib.kvsnap_pool_wait_many(pool, 1, _arrays([12345])[0]) == -1
    finally:
        lib.kvsnap_pool_destroy(pool)


def test_copy_many_merges_entries_adjacent_on_both_sides(lib):
    pool = lib.kvsnap_pool_create(96, 0)
    try:
        blocks = [reserve(lib, pool, 16) for _ in range(4)]      # reserved in a row: adjacent in the arena
        for k, (_, _, ptr) in enumerate(blocks):
            C.memmove(ptr, bytes([65 + k]) * 16, 16)
        device = C.create_string_buffer(80)
        dev = C.addressof(device)
        ids = [b[1] for b in blocks]
        # Device side adjacent for blocks 0-1 and 2-3, a 16-byte gap between them: two copies.
        arrays = _arrays(ids, [0, 0, 0, 0], [dev, dev + 16, dev + 48, dev + 64], [16] * 4)
        assert lib.kvsnap_pool_copy_many(pool, 4, *arrays, 0, 0) == 0
        assert lib.fake_cuda_pending() == 2
        assert lib.kvsnap_pool_wait_many(pool, 4, _arrays(ids)[0]) == 0
        assert device.raw == b"A" * 16 + b"B" * 16 + b"\0" * 16 + b"C" * 16 + b"D" * 16
        # Host side out of order: nothing merges.
        arrays = _arrays([ids[1], ids[0]], [0, 0], [dev, dev + 16], [16, 16])
        assert lib.kvsnap_pool_copy_many(pool, 2, *arrays, 1, 0) == 0
        assert lib.fake_cuda_pending() == 2
        assert lib.kvsnap_pool_wait_many(pool, 2, _arrays(ids[:2])[0]) == 0
    finally:
        lib.kvsnap_pool_destroy(pool)
