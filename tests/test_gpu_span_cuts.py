"""The device-memory kernels with spans cut into other units, against the oracle.

Pairs (KVSNAP_DP_PAIRS): when every span has one size S of 2 or 4 KiB (a TP-8
or TP-16 shard's) and the span count is even, the plane folds runs of units
that are pairs of consecutive spans: each lane owns 2 * S / 32 contiguous
packed bytes, lines 0..15 of a step lie in the pair's first span and lines
16..31 in its second.
Splits (KVSNAP_DP_SPLIT2 / SPLIT4): when every span has one size of 32 or
64 KiB (a Qwen3-8B layer's), units are 16 KiB pieces of a span, and each
piece's CRC is placed past the span's later pieces.
These cases cover each cut, token- and head-major storage, a ragged last
block (which is not split), and one or three CTAs, so that one warp walks many
units of many blocks. The oracle (oracle/oracle.py) gives the packed bytes,
the tail zeroing, the digests and the restored cache.
"""
import numpy as np
import pytest
import torch

import kvgen
from oracle import oracle

pytestmark = pytest.mark.gpu

BLOCKS, N = 10, 16

# name: (layers, heads, width in bf16 elements, token-major storage); S = heads * N * width * 2
SHAPES = {
    "s4k": (16, 1, 128, False),         # S = 4 KiB (a TP-8 shard's spans): pairs, 8 KiB units, 256 B a lane
    "s4k_tok": (6, 2, 64, True),        # the same size, token-major [B, N, H, C] storage
    "s2k": (8, 1, 64, False),           # S = 2 KiB: pairs, 4 KiB units, one line a lane
    "s32k": (3, 8, 128, True),          # S = 32 KiB (Qwen3-8B, token-major as vLLM stores it): halves
    "s32k_head": (4, 8, 128, False),    # the same size, head-major
    "s64k": (2, 16, 128, False),        # S = 64 KiB: quarters
}
CUT = {"s4k": "PAIRS", "s4k_tok": "PAIRS", "s2k": "PAIRS", "s32k": "SPLIT2", "s32k_head": "SPLIT2",
       "s64k": "SPLIT4"}


def build(shape):
    layers, h, c, token_major = SHAPES[shape]
    storages, views, caches, tensors = {}, {}, {}, {}
    per_block = h * N * c * 2
    for i in range(layers):
        name = f"layer.{i:02d}"
        buf = kvgen.random_bytes(9100 + 31 * i + layers, BLOCKS * per_block)
        storages[name] = buf
        stride = (c, h * c, 1) if token_major else (N * c, c, 1)
        views[name] = oracle.Span(name, name, 0, per_block, (h, N, c), stride, 2, BLOCKS)
        t = torch.from_numpy(buf.copy()).cuda()
        tensors[name] = t
        caches[name] = t.view(torch.bfloat16).as_strided((BLOCKS, h, N, c), (per_block // 2,) + stride)
    return storages, oracle.register(views, N), caches, tensors


@pytest.mark.parametrize("shape", sorted(SHAPES))
@pytest.mark.parametrize("ctas", [0, 1, 3])
@pytest.mark.parametrize("tokens", [6 * N, 5 * N + 3])
def test_span_cuts_save_and_restore(shape, ctas, tokens):
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    storages, layout, caches, tensors = build(shape)
    plane = TorchBlockDataPlane(caches, N, 64 << 20, save_mode="staged", restore_mode="staged", ctas=ctas)
    try:
        assert plane.block_bytes == layout.block_bytes
        plane.warm_up()
        assert plane._hbm & getattr(_abi, CUT[shape]), "spans of one size take their cut"
        assert bool(plane._hbm & _abi.RUNS) == (CUT[shape] == "PAIRS")
        saved = [7, 2, 9, 0, 4, 8][: (tokens + N - 1) // N]
        expected = oracle.pack(storages, layout, saved, tokens)
        size = plane.block_bytes
        staged = plane.pool.reserve(size * len(saved))
        targets = [(staged, i * size) for i in range(len(saved))]
        digests = []
        plane.save_gather(saved, targets, tokens, digests=digests)
        for i in range(len(saved)):
            assert staged.read_range(i * size, size) == expected[i].tobytes(), f"block {i}"
        assert [tuple(d) for d in digests] == [tuple(d) for d in oracle.digests(expected)]

        restored = [1, 5, 3, 6, 9, 0][: len(saved)]
        crcs = [oracle.crc32c(b) for b in expected]
        plane.load_scatter(restored, targets, expected_crc32c=crcs)
        oracle.unpack(storages, layout, restored, expected)
        torch.cuda.synchronize()
        for name, t in tensors.items():
            assert np.array_equal(t.cpu().numpy(), storages[name]), name
        staged.close()
    finally:
        plane.close()


def _raw(plane, ids, flags, mode="gather", sources=None):
    """kvsnap_dp_gather (or _scatter from ``sources``) of whole blocks with explicit flags.

    Returns (rc, status, packed bytes, crc list)."""
    from kvsnap_b200.dataplane import _dp
    lib = _dp(plane.pool.lib)
    n, size = len(ids), plane.block_bytes
    packed = torch.zeros(n * size, dtype=torch.uint8, device="cuda")
    if sources is not None:
        packed.copy_(torch.from_numpy(sources))
    table = torch.tensor([packed.data_ptr() + i * size for i in range(n)], dtype=torch.int64, device="cuda")
    blocks = torch.tensor(ids, dtype=torch.int64, device="cuda")
    crc = torch.zeros(n, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    spans, stream = plane._spans(), torch.cuda.current_stream().cuda_stream
    if mode == "gather":
        rc = lib.kvsnap_dp_gather(spans.data_ptr(), len(plane.layers), size, blocks.data_ptr(), table.data_ptr(),
                                  n, 0, crc.data_ptr(), status.data_ptr(), flags, 0, stream)
    else:
        rc = lib.kvsnap_dp_scatter(spans.data_ptr(), len(plane.layers), size, table.data_ptr(), blocks.data_ptr(),
                                   n, crc.data_ptr(), 0, 0, status.data_ptr(), flags, 0, stream)
    torch.cuda.synchronize()
    return rc, int(status.item()), packed.cpu().numpy(), [v & 0xFFFFFFFF for v in crc.tolist()]


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_cuts_match_runs_and_single_spans(shape):
    """The same bytes and CRCs with each cut the spans allow, with runs and with whole spans, both ways."""
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    storages, layout, caches, tensors = build(shape)
    plane = TorchBlockDataPlane(caches, N, 64 << 20)
    try:
        plane.warm_up()
        ids = [3, 8, 1, 6, 0]
        want = oracle.pack(storages, layout, ids, len(ids) * N)
        crcs = [oracle.crc32c(b) for b in want]
        flat = np.concatenate(want)
        size = layout.spans[0].bytes
        cuts = [("spans", 16 | _abi.HBM), ("runs", 16 | _abi.HBM | _abi.RUNS)]
        if size in _abi.PAIR_SPAN_BYTES:
            cuts.append(("pairs", 16 | _abi.HBM | _abi.RUNS | _abi.PAIRS))
        cuts += [(f"split{k}", 16 | _abi.HBM | flag) for k, flag in ((2, _abi.SPLIT2), (4, _abi.SPLIT4))
                 if size % (k * 4096) == 0]
        assert len(cuts) > 2
        for name, flags in cuts:
            rc, status, out, crc = _raw(plane, ids, flags)
            assert rc == 0 and status == 0, name
            assert out.tobytes() == flat.tobytes() and crc == crcs, name
            rc, status, _, crc = _raw(plane, [9, 2, 5, 7, 4], flags, mode="scatter", sources=flat)
            assert rc == 0 and status == 0 and crc == crcs, name
        oracle.unpack(storages, layout, [9, 2, 5, 7, 4], want)
        torch.cuda.synchronize()
        for name, t in tensors.items():
            assert np.array_equal(t.cpu().numpy(), storages[name]), name
    finally:
        plane.close()


def test_pair_of_spans_of_two_sizes_is_flagged_not_moved():
    """Under KVSNAP_DP_PAIRS, a pair whose spans differ sets KVSNAP_DP_BAD_CUT and is not written,
    while the valid pairs of the same launch are; an odd span count, or a split with runs, is
    refused on the host."""
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import TorchBlockDataPlane

    def plane_of(heads):
        caches = {}
        for i, h in enumerate(heads):
            per_block = h * N * 128 * 2
            t = torch.from_numpy(kvgen.random_bytes(77 + i, BLOCKS * per_block)).cuda()
            caches[f"layer.{i}"] = t.view(torch.bfloat16).as_strided((BLOCKS, h, N, 128),
                                                                     (per_block // 2, N * 128, 128, 1))
        return TorchBlockDataPlane(caches, N, 64 << 20)

    plane = plane_of((1, 1, 1, 2))                   # pairs (4, 4) KiB and (4, 8) KiB
    try:
        plane.warm_up()
        assert plane._hbm & _abi.RUNS and not plane._hbm & _abi.PAIRS, "spans of two sizes do not pair"
        flags = 16 | _abi.HBM | _abi.RUNS | _abi.PAIRS
        rc, status, out, _ = _raw(plane, [2, 5], flags)
        assert rc == 0 and status & _abi.BAD_CUT
        size = plane.block_bytes
        for i, block in enumerate((2, 5)):
            first = plane.caches["layer.0"][block].contiguous().view(torch.uint8).cpu().numpy().ravel()
            assert out[i * size: i * size + 4096].tobytes() == first.tobytes(), "the valid pair is moved"
            assert not out[i * size + 8192: (i + 1) * size].any(), "the mismatched pair is not"
    finally:
        plane.close()
    plane = plane_of((1, 1, 1))
    try:
        plane.warm_up()
        rc, _, _, _ = _raw(plane, [2, 5], 16 | _abi.HBM | _abi.RUNS | _abi.PAIRS)
        assert rc != 0 and b"even" in plane.pool.lib.kvsnap_cuda_error()
        rc, _, _, _ = _raw(plane, [2, 5], 16 | _abi.HBM | _abi.RUNS | _abi.SPLIT2)
        assert rc != 0 and b"split" in plane.pool.lib.kvsnap_cuda_error()
    finally:
        plane.close()


def test_split_that_leaves_padded_pieces_is_flagged_not_moved():
    """SPLIT2 on 34 KiB spans (17 KiB pieces, not whole lines a lane) sets KVSNAP_DP_BAD_CUT and
    writes nothing."""
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    caches = {}
    for i in range(2):
        per_block = 8 * N * 136 * 2
        t = torch.from_numpy(kvgen.random_bytes(99 + i, BLOCKS * per_block)).cuda()
        caches[f"layer.{i}"] = t.view(torch.bfloat16).as_strided((BLOCKS, 8, N, 136),
                                                                 (per_block // 2, N * 136, 136, 1))
    plane = TorchBlockDataPlane(caches, N, 64 << 20)
    try:
        plane.warm_up()
        assert not plane._hbm & (_abi.SPLIT2 | _abi.SPLIT4), "34 KiB spans are not split"
        rc, status, out, _ = _raw(plane, [4, 1], 16 | _abi.HBM | _abi.SPLIT2)
        assert rc == 0 and status & _abi.BAD_CUT and not out.any()
    finally:
        plane.close()
