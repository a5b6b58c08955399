"""The device-memory kernels on spans of uneven sizes, against the oracle.

The save gather and restore scatter between HBM buffers split each (block,
span) unit into 32 equal lane segments of whole 128-byte lines, front-padded
with zeros. The golden geometries all have 32 KiB spans, where that padding is
empty. These layers make it non-empty and uneven:
- 512-byte spans, padded to 4 KiB, so most lanes carry only zeros;
- 3840-byte spans (one line of padding);
- 34816-byte spans (nine lines a lane, half a segment of padding).

They also mix token-major storage ([B,N,H,C] under a [B,H,N,C] view) with
head-major storage, and a 24-byte row that the tail mask handles byte by byte.
With a single CTA, one warp meets units of every size in turn, so the
per-size lane shift must be recomputed whenever the size changes. The "small"
set has only spans of at most 8 KiB, which the plane launches with
KVSNAP_DP_RUNS: a warp folds a block's consecutive spans as one run, and
spans of a size other than the first one's take the multiply fallback.
The oracle (oracle/oracle.py) gives the packed bytes, the tail zeroing, the
digests and the restored cache.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import kvgen
from oracle import oracle

pytestmark = pytest.mark.gpu

BLOCKS, N = 12, 16
# name: (heads, width in bf16 elements, token-major storage)
LAYERS = {
    "layer.a": (2, 8, True),        # 512 B
    "layer.b": (3, 40, False),      # 3840 B
    "layer.c": (8, 136, True),      # 34816 B
    "layer.d": (5, 12, False),      # 1920 B, 24-byte rows
}


SETS = {"mixed": sorted(LAYERS), "small": ["layer.a", "layer.b", "layer.d"]}


def build(names):
    storages, views, caches, tensors = {}, {}, {}, {}
    for i, name in enumerate(names):
        h, c, token_major = LAYERS[name]
        per_block = h * N * c * 2
        buf = kvgen.random_bytes(7000 + i, BLOCKS * per_block)
        storages[name] = buf
        if token_major:      # storage [B, N, H, C], view [B, H, N, C]
            stride = (c, h * c, 1)
        else:                # storage [B, H, N, C]
            stride = (N * c, c, 1)
        views[name] = oracle.Span(name, name, 0, per_block, (h, N, c), stride, 2, BLOCKS)
        t = torch.from_numpy(buf.copy()).cuda()
        tensors[name] = t
        caches[name] = t.view(torch.bfloat16).as_strided((BLOCKS, h, N, c), (per_block // 2,) + stride)
    return storages, oracle.register(views, N), caches, tensors


@pytest.mark.parametrize("layer_set", ["mixed", "small"])
@pytest.mark.parametrize("ctas", [0, 1, 3])
@pytest.mark.parametrize("tokens", [5 * N, 4 * N + 5, 1 * N + 1, 3])
def test_uneven_spans_save_and_restore(layer_set, ctas, tokens):
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    storages, layout, caches, tensors = build(SETS[layer_set])
    plane = TorchBlockDataPlane(caches, N, 64 << 20, save_mode="staged", restore_mode="staged", ctas=ctas)
    try:
        assert plane.block_bytes == layout.block_bytes
        plane.warm_up()
        assert plane._hbm, "these layers must take the device-memory kernels"
        assert bool(plane._hbm & _abi.RUNS) == (layer_set == "small")
        saved = [7, 2, 9, 0, 11][: (tokens + N - 1) // N]
        expected = oracle.pack(storages, layout, saved, tokens)
        size = plane.block_bytes
        staged = plane.pool.reserve(size * len(saved))
        targets = [(staged, i * size) for i in range(len(saved))]
        digests = []
        plane.save_gather(saved, targets, tokens, digests=digests)
        for i in range(len(saved)):
            assert staged.read_range(i * size, size) == expected[i].tobytes(), f"block {i}"
        assert [tuple(d) for d in digests] == [tuple(d) for d in oracle.digests(expected)]

        restored = [1, 4, 10, 3, 8][: len(saved)]
        crcs = [oracle.crc32c(b) for b in expected]
        plane.load_scatter(restored, targets, expected_crc32c=crcs)
        oracle.unpack(storages, layout, restored, expected)
        torch.cuda.synchronize()
        for name, t in tensors.items():
            assert np.array_equal(t.cpu().numpy(), storages[name]), name
        staged.close()
    finally:
        plane.close()


def test_device_crc_of_uneven_lengths_with_one_cta():
    """kvsnap_dp_crc32c over device blocks whose 64 KiB pieces end in short, padded segments."""
    from kvsnap_b200.dataplane import _dp, _load
    lib = _dp(_load())
    for length in (16, 4080, 4096 + 16, 65536 + 4096 + 48, 3 * 65536 + 2048):
        n = 3
        data = [kvgen.random_bytes(50 + length + i, length) for i in range(n)]
        buf = torch.from_numpy(np.concatenate(data)).cuda()
        addrs = torch.tensor([buf.data_ptr() + i * length for i in range(n)], dtype=torch.int64, device="cuda")
        crc = torch.empty(n, dtype=torch.int32, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        assert lib.kvsnap_dp_crc32c(addrs.data_ptr(), n, length, crc.data_ptr(), 0, status.data_ptr(),
                                    16 | 0x100, 1, s) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert [v & 0xFFFFFFFF for v in crc.tolist()] == [oracle.crc32c(d.tobytes()) for d in data], length
