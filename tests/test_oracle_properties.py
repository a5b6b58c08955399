"""Property tests (CPU) of the CRC32C algebra the GPU kernels rely on, and of the oracle itself.

The kernels never compute a block's CRC32C front to back: they CRC pieces anywhere in the
block, in lanes, and combine raw registers by multiplying with powers of x. These properties
state that arithmetic on random inputs, against the oracle's C restatement of the reference's
CRC32C (oracle/crc32c.c, itself pinned to the reference's vectors in test_oracle_golden.py):
- linearity and the combine rule, incremental extension, table against bitwise;
- the per-unit placement and the finish step's constant (kvsnap_b200/csrc/dataplane.cu:
  each unit's raw register times x^(8 * bytes after it), XORed, then
  ~0 ^ ~0 * x^(8 * block_bytes));
- the segment lanes of the device-memory kernels, for random segment sizes and padding;
- the oracle's pack / unpack round trip and tail zeroing on random small layouts;
- the unit-cut flags the plane picks, for random span-size lists.
"""
import numpy as np
from hypothesis import given, settings, strategies as st

from oracle import oracle

SETTINGS = settings(max_examples=60, deadline=None)


def raw(data: bytes) -> int:
    """The raw CRC register of data (no initial or final inversion)."""
    return ~oracle.crc32c(data, 0xFFFFFFFF) & 0xFFFFFFFF


@SETTINGS
@given(st.binary(max_size=3000), st.binary(max_size=3000))
def test_combine_rule_and_incremental_extension(a, b):
    whole = oracle.crc32c(a + b)
    assert oracle.crc32c_combine(oracle.crc32c(a), oracle.crc32c(b), len(b)) == whole
    assert oracle.crc32c(b, oracle.crc32c(a)) == whole
    assert raw(a + b) == oracle.gf_mulmod(raw(a), oracle.xpow8n(len(b))) ^ raw(b)


@SETTINGS
@given(st.binary(max_size=2000))
def test_table_crc_equals_bitwise(data):
    assert oracle.crc32c(data) == oracle.crc32c_bitwise(data)


@SETTINGS
@given(st.binary(min_size=1, max_size=6000), st.lists(st.integers(0, 6000), max_size=6))
def test_units_placed_anywhere_and_finished_give_the_block_crc(block, cuts):
    """Cut a block at random points into units, in any order: XOR of raw(unit) * x^(8 * bytes
    after it), plus the finish constant, is the block's CRC32C."""
    points = sorted({0, len(block), *[c % (len(block) + 1) for c in cuts]})
    units = list(zip(points, points[1:]))
    acc = 0
    for start, end in reversed(units):            # order does not matter: XOR
        acc ^= oracle.gf_mulmod(raw(block[start:end]), oracle.xpow8n(len(block) - end))
    init = 0xFFFFFFFF ^ oracle.gf_mulmod(0xFFFFFFFF, oracle.xpow8n(len(block)))
    assert acc ^ init == oracle.crc32c(block)


@settings(max_examples=12, deadline=None)
@given(st.sampled_from([1024, 2048]), st.integers(0, 1023), st.integers(0, 2 ** 32 - 1))
def test_segment_lanes_on_random_units(seg, pad, seed):
    """Four segments of `seg` bytes, front-padded by `pad`; eight lanes a segment, four chains a
    lane folding a word then 124 bytes; Horner over chains, the lane's place, XOR over lanes:
    raw(unit) * x^(8 * 124)."""
    unit = np.random.default_rng(seed).integers(0, 256, 4 * seg - pad, dtype=np.uint8).tobytes()
    padded = bytes(pad) + unit
    line, x32 = oracle.xpow8n(128), oracle.xpow8n(4)
    total = 0
    for lane in range(32):
        r, s = lane >> 3, lane & 7
        c = [0, 0, 0, 0]
        for ln in range(seg // 128):
            at = r * seg + ln * 128 + 16 * s
            for k in range(4):
                c[k] = oracle.gf_mulmod(c[k] ^ int.from_bytes(padded[at + 4 * k:at + 4 * k + 4], "little"), line)
        h = oracle.gf_mulmod(oracle.gf_mulmod(oracle.gf_mulmod(c[0], x32) ^ c[1], x32) ^ c[2], x32) ^ c[3]
        total ^= oracle.gf_mulmod(h, oracle.xpow8n(16 * (7 - s) + seg * (3 - r)))
    assert total == oracle.gf_mulmod(raw(unit), oracle.xpow8n(124))


@SETTINGS
@given(st.integers(1, 4), st.integers(1, 3), st.integers(1, 5), st.booleans(),
       st.integers(1, 6), st.integers(0, 2 ** 32 - 1))
def test_pack_unpack_round_trip_and_tail(layers, heads, width, token_major, nblocks, seed):
    """pack then unpack into other blocks restores every packed span; tail zeroing touches only
    the last block's token slots at or past the valid count."""
    n_tok, blocks = 4, 8
    rng = np.random.default_rng(seed)
    storages, views = {}, {}
    per_block = heads * n_tok * width * 2
    for i in range(layers):
        name = f"l{i}"
        storages[name] = rng.integers(0, 256, blocks * per_block, dtype=np.uint8)
        stride = (width, heads * width, 1) if token_major else (n_tok * width, width, 1)
        views[name] = oracle.Span(name, name, 0, per_block, (heads, n_tok, width), stride, 2, blocks)
    layout = oracle.register(views, n_tok)
    ids = list(rng.permutation(blocks)[:nblocks])
    tokens = int(rng.integers((nblocks - 1) * n_tok + 1, nblocks * n_tok + 1))
    full = oracle.pack(storages, layout, ids, nblocks * n_tok)
    packed = oracle.pack(storages, layout, ids, tokens)
    for a, b in zip(full[:-1], packed[:-1]):
        assert np.array_equal(a, b)
    valid = tokens % n_tok
    changed = np.flatnonzero(full[-1] != packed[-1])
    assert valid or changed.size == 0
    assert not packed[-1][changed].any(), "only zeroed bytes differ"
    copy = {k: v.copy() for k, v in storages.items()}
    targets = [int(x) for x in rng.permutation(blocks)[:nblocks]]
    oracle.unpack(copy, layout, targets, packed)
    again = oracle.pack(copy, layout, targets, nblocks * n_tok)
    for a, b in zip(packed, again):
        assert np.array_equal(a, b)


@SETTINGS
@given(st.lists(st.sampled_from([512, 1920, 2048, 4096, 8192, 16384, 32768, 34816, 65536]),
                min_size=1, max_size=12),
       st.sampled_from([16, 8]))
def test_unit_cut_flags_are_consistent(spans, vec):
    from kvsnap_b200 import _abi
    flags = _abi.hbm_flags(spans, vec)
    if vec != 16:
        assert flags == 0
        return
    assert flags & _abi.HBM
    one = len(set(spans)) == 1
    assert bool(flags & _abi.RUNS) == (max(spans) <= _abi.RUNS_SPAN_BYTES)
    if flags & _abi.PAIRS:
        assert flags & _abi.RUNS and one and spans[0] in _abi.PAIR_SPAN_BYTES and len(spans) % 2 == 0
    if flags & (_abi.SPLIT2 | _abi.SPLIT4):
        assert one and not flags & _abi.RUNS
        pieces = 2 if flags & _abi.SPLIT2 else 4
        assert spans[0] == pieces * _abi.SPLIT_PIECE_BYTES


def test_full_size_generators_reproduce_the_fixture_stream():
    """The GPU fill (torch int64 splitmix64) and the lazy host slices give kvgen.random_bytes' bytes exactly,
    so the full-size GPU tests feed the CUDA path and the oracle the same cache."""
    import torch
    import kvgen
    seed, nbytes = 28011, (1 << 18) + 24
    want = kvgen.random_bytes(seed, nbytes)
    buf = torch.empty(nbytes, dtype=torch.uint8)
    kvgen.fill_random(buf, seed, chunk_words=1 << 12)
    assert np.array_equal(buf.numpy(), want)
    lazy = kvgen.LazyBytes(seed, nbytes)
    for start, stop in [(0, 8), (3, 1000), (4096, 8192), (nbytes - 13, nbytes), (77, 77), (0, nbytes)]:
        assert np.array_equal(lazy[start:stop], want[start:stop])


def test_dedup_from_precomputed_digests_is_the_dedup_rule():
    import kvgen
    blocks = [kvgen.random_bytes(s, 4096) for s in (1, 2, 1, 3, 2)]
    unique, segments = oracle.dedup(blocks)
    assert oracle.dedup_digests(oracle.digests(blocks), [len(b) for b in blocks]) == (unique, segments)
    assert len(unique) == 3 and [s["first_block"] for s in segments] == [0, 1, 2, 3, 4]
