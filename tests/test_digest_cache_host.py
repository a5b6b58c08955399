"""DigestCache (kvsnap_b200/dataplane.py) bookkeeping, on the CPU.

The cache's GPU use (a save hashing only the blocks it has not seen under their
generation) is tested in tests/test_gpu_parity.py; here: keys are (block,
generation), the least recently used entries go first, forget drops every
generation of a block, and bad digests are refused.
"""
import pytest


def sha(k):
    return f"{k:064x}"


def test_entries_are_keyed_by_block_and_generation():
    from kvsnap_b200.dataplane import DigestCache
    cache = DigestCache(capacity=3)
    cache.put(7, 1, (sha(1), 11))
    assert cache.get(7, 1) == (sha(1), 11)
    assert cache.get(7, 2) is None and cache.get(8, 1) is None
    cache.put(7, 2, (sha(2), -1))                    # CRCs are stored as unsigned 32-bit values
    assert cache.get(7, 2) == (sha(2), 0xFFFFFFFF)


def test_least_recently_used_go_first_and_forget_drops_all_generations():
    from kvsnap_b200.dataplane import DigestCache
    cache = DigestCache(capacity=3)
    for block in range(3):
        cache.put(block, 0, (sha(block), block))
    cache.get(0, 0)                                  # 0 is now the most recently used
    cache.put(3, 0, (sha(3), 3))
    assert cache.get(1, 0) is None and cache.get(0, 0) is not None and len(cache) == 3
    cache.put(0, 5, (sha(9), 9))
    cache.forget([0])
    assert cache.get(0, 0) is None and cache.get(0, 5) is None and cache.get(3, 0) is not None


def test_bad_arguments_are_refused():
    from kvsnap_b200.dataplane import DigestCache
    with pytest.raises(ValueError):
        DigestCache(capacity=0)
    with pytest.raises(ValueError):
        DigestCache().put(1, 1, ("abc", 1))
