"""Incremental Castagnoli CRC32C on the host, a drop-in for ``kvsnap.store.crc32c.crc32c``.

Same contract as the reference (kvsnap/store/crc32c.py:17-27): ``crc32c(data, crc=0)``
with ``crc`` a prior value in [0, 2**32), computed by the native library
(include/kvsnap_io.h ``kvsnap_crc32c_extend``).
"""
from __future__ import annotations

from .native_io import get_io_backend


def crc32c(data: bytes, crc: int = 0) -> int:
    """Return CRC32C; passing a prior CRC permits incremental checksumming."""
    if type(crc) is not int or not 0 <= crc <= 0xFFFFFFFF:
        raise ValueError("prior CRC32C must fit uint32")
    return get_io_backend().crc32c(data, crc)
