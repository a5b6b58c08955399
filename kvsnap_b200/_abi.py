"""ctypes declarations of include/kvsnap_cuda.h and include/kvsnap_io.h.

Kept in one place so the pool, the data plane, the tests and the bench bind the
same prototypes. Loading never initialises CUDA; a missing or mismatched
library raises, there is no fallback.
"""
from __future__ import annotations

import ctypes as C

DP_ABI_VERSION = 1
POOL_ABI_VERSION = 2
IO_ABI_VERSION = 1

MISALIGNED, BAD_BLOCK, CRC_MISMATCH, BAD_CUT = 1, 2, 4, 8
# OR into a kernel's `vec` when every packed address is device memory.
HBM = 0x100
RUNS = 0x200            # with HBM: spans of at most RUNS_SPAN_BYTES fold in runs
RUNS_SPAN_BYTES = 8 << 10
PAIRS = 0x400           # with RUNS: spans all of one size in PAIR_SPAN_BYTES, an even count: units of two spans
PAIR_SPAN_BYTES = (2 << 10, 4 << 10)
SPLIT2, SPLIT4 = 0x800, 0x1000   # with HBM, without RUNS: units of 1/2 or 1/4 of a span
CRC_ACCUMULATE = 0x2000          # with HBM: add to the CRC accumulators, leave them raw (kvsnap_dp_crc32c_finish)
SPLIT_PIECE_BYTES = 16 << 10     # the unit size the plane splits large spans of one size into


def split_flag(span_bytes):
    """The KVSNAP_DP_SPLIT* flag that cuts spans of ``span_bytes`` into SPLIT_PIECE_BYTES, or 0."""
    return {2: SPLIT2, 4: SPLIT4}.get(span_bytes // SPLIT_PIECE_BYTES, 0) if span_bytes % SPLIT_PIECE_BYTES == 0 else 0


def hbm_flags(span_bytes, vec):
    """The flags a device-to-device gather or scatter of these spans takes beside ``vec``.

    0 unless vec is 16. Otherwise KVSNAP_DP_HBM and the unit cut that measured fastest on B200:
    spans all of at most RUNS_SPAN_BYTES fold in runs (2 and 4 KiB spans of one size, an even
    count, in pairs); spans of one size of 32 or 64 KiB move in 16 KiB pieces; others whole.
    """
    if vec != 16 or not span_bytes:
        return 0
    flags = HBM
    sizes = set(span_bytes)
    one_size = next(iter(sizes)) if len(sizes) == 1 else 0
    if max(span_bytes) <= RUNS_SPAN_BYTES:
        flags |= RUNS
        if one_size in PAIR_SPAN_BYTES and len(span_bytes) % 2 == 0:
            flags |= PAIRS
    elif one_size:
        flags |= split_flag(one_size)
    return flags


class Span(C.Structure):
    """``kvsnap_span``: one registered layer view (64 bytes)."""
    _fields_ = [("base", C.c_int64), ("pitch", C.c_int64), ("offset", C.c_int64), ("bytes", C.c_int64),
                ("token_pitch", C.c_int64), ("tokens", C.c_int32), ("row_bytes", C.c_int32),
                ("nblocks", C.c_int64), ("crc_shift", C.c_uint32), ("flags", C.c_uint32)]


assert C.sizeof(Span) == 64

_P = C.c_void_p
_I64 = C.c_int64
_U64 = C.c_uint64
_SZ = C.c_size_t

POOL_API = {
    "kvsnap_pool_abi_version": ([], C.c_int),
    "kvsnap_cuda_error": ([], C.c_char_p),
    "kvsnap_pool_create": ([_SZ, C.c_int], _P),
    "kvsnap_pool_destroy": ([_P], None),
    "kvsnap_pool_close_checked": ([_P], C.c_int),
    "kvsnap_pool_copy_stream": ([_P, C.POINTER(C.c_size_t)], C.c_int),
    "kvsnap_pool_reserve": ([_P, _SZ, C.POINTER(C.c_uint64), C.POINTER(C.c_void_p)], C.c_int),
    "kvsnap_pool_copy": ([_P, C.c_uint64, _SZ, _P, _SZ, C.c_int, _SZ], C.c_int),
    "kvsnap_pool_copy_2d": ([_P, C.c_uint64, _SZ, _SZ, _P, _SZ, _SZ, _SZ, C.c_int, _SZ], C.c_int),
    "kvsnap_pool_wait": ([_P, C.c_uint64], C.c_int),
    "kvsnap_pool_ready": ([_P, C.c_uint64], C.c_int),
    "kvsnap_pool_release": ([_P, C.c_uint64], C.c_int),
}

# Pool entry points this library adds to the reference's ABI 2 set.
POOL_EXTRA = {
    "kvsnap_pool_mark": ([_P, C.c_uint64, _SZ], C.c_int),
    "kvsnap_pool_copy_on": ([_P, C.c_uint64, _SZ, _P, _SZ, C.c_int, _SZ], C.c_int),
    "kvsnap_pool_copy_many": ([_P, C.c_int64, _P, _P, _P, _P, C.c_int, _SZ], C.c_int),
    "kvsnap_pool_wait_many": ([_P, C.c_int64, _P], C.c_int),
    "kvsnap_pool_create_shared": ([_SZ, C.c_int, C.c_char_p], _P),
    "kvsnap_pool_arena": ([_P, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)], C.c_int),
    "kvsnap_shared_open": ([C.c_char_p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)], C.c_int),
    "kvsnap_shared_close": ([_P, _SZ], C.c_int),
}

DP_API = {
    "kvsnap_dp_abi_version": ([], C.c_int),
    "kvsnap_dp_plan": ([C.POINTER(Span), C.c_int, C.POINTER(C.c_uint64)], C.c_int),
    "kvsnap_dp_crc32c_host": ([_P, _SZ, C.c_uint32], C.c_uint32),
    "kvsnap_dp_gather": ([_P, C.c_int, _U64, _P, _P, _I64, C.c_int32, _P, _P, C.c_int, C.c_int, _SZ], C.c_int),
    "kvsnap_dp_scatter": ([_P, C.c_int, _U64, _P, _P, _I64, _P, _P, _P, _P, C.c_int, C.c_int, _SZ], C.c_int),
    "kvsnap_dp_crc32c": ([_P, _I64, _U64, _P, _P, _P, C.c_int, C.c_int, _SZ], C.c_int),
    "kvsnap_dp_sha256": ([_P, _I64, _U64, _P, _SZ], C.c_int),
    "kvsnap_dp_sha256_part": ([_P, _I64, _U64, _U64, _U64, _P, _P, _SZ], C.c_int),
    "kvsnap_dp_crc32c_finish": ([_P, _P, _I64, _U64, _P, _SZ], C.c_int),
    "kvsnap_dp_land": ([_P, _I64, _P, _I64, _I64, _I64, _P, C.c_int, _SZ], C.c_int),
    "kvsnap_dp_land_strided": ([_P, _I64, _P, _I64, _I64, _I64, _SZ], C.c_int),
    "kvsnap_dp_copy_host_blocks": ([_P, _P, _I64, _P, _P, _P, _P, _I64, C.c_int, _SZ], C.c_int),
    "kvsnap_dp_regroup": ([_P, _P, C.c_int, _P, C.c_int, _P, _I64, _P, C.c_int, _SZ], C.c_int),
    "kvsnap_dp_device_alloc": ([_SZ, C.c_int, C.POINTER(C.c_void_p)], C.c_int),
    "kvsnap_dp_device_free": ([_P], C.c_int),
    "kvsnap_dp_ipc_export": ([_P, _P], C.c_int),
    "kvsnap_dp_ipc_open": ([_P, C.c_int, C.POINTER(C.c_void_p)], C.c_int),
    "kvsnap_dp_ipc_close": ([_P], C.c_int),
    "kvsnap_dp_scatter_verify_static": ([_P, C.c_int, _U64, _P, _P, _I64, _P, _P, C.c_int, C.c_int, _SZ], C.c_int),
}

# Blocks the no-allocation verified scatter handles in one call (include/kvsnap_cuda.h).
STATIC_MAX_BLOCKS = 65536

IO_API = {
    "kvsnap_io_abi_version": ([], C.c_int),
    "kvsnap_crc32c_extend": ([_P, _SZ, C.c_uint32], C.c_uint32),
    "kvsnap_crc32c": ([_P, _SZ], C.c_uint32),
    "kvsnap_pwrite_all": ([C.c_int, _P, _SZ, C.c_int64, C.c_int], C.c_int),
    "kvsnap_pread_all": ([C.c_int, _P, _SZ, C.c_int64], C.c_int),
    "kvsnap_io_pool_create": ([_SZ, _SZ], _P),
    "kvsnap_io_pool_destroy": ([_P], None),
    "kvsnap_io_pool_transfer": ([_P, C.c_int, _P, _SZ, C.c_int64, C.c_int, C.c_int], C.c_int),
}


def declare(lib, api: dict, *, required: bool = True):
    """Set argtypes/restype; a symbol missing from the library raises when ``required``."""
    for name, (args, result) in api.items():
        try:
            fn = getattr(lib, name)
        except AttributeError:
            if required:
                raise RuntimeError(f"{lib._name}: missing symbol {name}; rebuild with python -m kvsnap_b200.build")
            continue
        fn.argtypes, fn.restype = args, result
    return lib


_cache = {}


def load(path, api: dict):
    """Load a library once per path and declare ``api`` on it."""
    key = str(path)
    if key not in _cache:
        _cache[key] = declare(C.CDLL(key), api)
    return _cache[key]
