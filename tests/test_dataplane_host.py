"""Host-side logic of the data plane on a CPU: the C ABI's exports, registration, and the span plan.

No kernel runs here. Registration runs on CPU tensors that report a CUDA
device (as the reference's own layout tests do), with the pinned pool
replaced by a mock. Its results must equal what the reference recorded
(tests/golden/golden.json): accept/reject, the ``layers`` metadata that
becomes the snapshot identity, and ``block_bytes``. The span plan and the way
the CUDA kernels combine partial CRCs are checked against the oracle.
"""
import ctypes as C
import re
from pathlib import Path
from types import SimpleNamespace
from unittest.mock import patch

import numpy as np
import pytest
import torch

from cases import GOLDEN, golden_case
from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]


class OnCuda:
    """A CPU tensor that reports a CUDA device, for registration's device check."""
    device = SimpleNamespace(type="cuda", index=0)

    def __init__(self, tensor):
        self._tensor = tensor

    def __getattr__(self, name):
        return getattr(self._tensor, name)

    def __getitem__(self, index):
        item = self._tensor[index]
        return OnCuda(item) if isinstance(item, torch.Tensor) and item.ndim >= 3 else item

    def permute(self, *dims):
        return OnCuda(self._tensor.permute(*dims))


def register(caches, block_size=16):
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    with patch("kvsnap_b200.dataplane.CudaPool"):
        return TorchBlockDataPlane({k: OnCuda(v) for k, v in caches.items()}, block_size, 1 << 20)


def declared(header):
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvsnap_\w+)\s*\(", text)))


def test_every_declared_entry_point_is_exported():
    from kvsnap_b200 import build
    cuda = C.CDLL(str(build.build_cuda()))
    io = C.CDLL(str(build.build_io()))
    cuda_symbols = declared("kvsnap_cuda.h")
    io_symbols = declared("kvsnap_io.h")
    assert "kvsnap_pool_reserve" in cuda_symbols and "kvsnap_dp_gather" in cuda_symbols
    assert "kvsnap_crc32c_extend" in io_symbols
    for name in cuda_symbols:
        assert hasattr(cuda, name), name
    for name in io_symbols:
        assert hasattr(io, name), name


def test_python_flag_constants_equal_the_header():
    """Every KVSNAP_DP_* flag and status bit the ctypes layer uses has the header's value."""
    from kvsnap_b200 import _abi
    text = (Path(__file__).resolve().parents[1] / "include" / "kvsnap_cuda.h").read_text()
    defines = {m.group(1): int(m.group(2), 0)
               for m in re.finditer(r"#define KVSNAP_DP_(\w+) (0x[0-9A-Fa-f]+|\d+)u?\b", text)}
    for name in ("MISALIGNED", "BAD_BLOCK", "CRC_MISMATCH", "BAD_CUT", "HBM", "RUNS", "PAIRS", "SPLIT2", "SPLIT4",
                 "CRC_ACCUMULATE"):
        assert getattr(_abi, name) == defines[name], name
    assert defines["SPLIT_MASK"] == _abi.SPLIT2 | _abi.SPLIT4
    assert defines["ABI_VERSION"] == _abi.DP_ABI_VERSION


def test_abi_versions_and_span_layout_load_without_a_gpu():
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import _dp, _load
    lib = _dp(_load())
    assert lib.kvsnap_pool_abi_version() == _abi.POOL_ABI_VERSION == 2
    assert lib.kvsnap_dp_abi_version() == _abi.DP_ABI_VERSION
    assert C.sizeof(_abi.Span) == 64
    for data in (b"", b"123456789", bytes(range(256)) * 9):
        assert lib.kvsnap_dp_crc32c_host(data, len(data), 0) == oracle.crc32c(data)
    assert lib.kvsnap_dp_crc32c_host(b"456789", 6, oracle.crc32c(b"123")) == 0xE3069283


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    from kvsnap_b200.dataplane import CudaPool
    monkeypatch.setenv("KVSNAP_CUDA_LIBRARY", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="not found"):
        CudaPool(1 << 20)


@pytest.mark.parametrize("row", GOLDEN["registration"], ids=lambda r: str(r["strides"]))
def test_registration_matches_the_reference(row):
    storage = torch.zeros(5 * max(row["strides"][0], 96) + 256, dtype=torch.bfloat16)
    cache = storage.as_strided((5, 3, 4, 8), row["strides"])
    if row["accepted"]:
        plane = register({"layer.0": cache}, 4)
        assert plane.block_bytes == row["block_bytes"]
        assert plane.layers == row["layers"]
    else:
        with pytest.raises(ValueError):
            register({"layer.0": cache}, 4)


def test_registration_rejects_what_the_reference_rejects():
    with pytest.raises(ValueError, match="empty"):
        register({})
    bad = torch.zeros((4, 8, 16, 128), dtype=torch.bfloat16).permute(0, 1, 3, 2)   # C not contiguous
    with pytest.raises(ValueError, match="unsupported KV layout"):
        register({"x": bad})
    with pytest.raises(ValueError, match="unsupported KV layout"):
        register({"x": torch.zeros((4, 8, 8, 128), dtype=torch.bfloat16)})           # N != block size


def cpu_caches(key):
    case, storages, _ = golden_case(key)
    if case["kind"] == "5d":
        return case, {name: torch.from_numpy(buf).view(torch.bfloat16).view(2, case["num_blocks"], 16, 8, 128)
                      for name, buf in storages.items()}
    view = torch.from_numpy(storages["backing"]).view(torch.bfloat16).view(case["num_layers"], case["num_blocks"],
                                                                           16, 8, 256)
    return case, {f"model.layers.{i}.self_attn.attn": view[i].permute(0, 2, 1, 3) for i in range(case["num_layers"])}


@pytest.mark.parametrize("key", ["vllm031", "qwen3_1p7b_5d", "qwen3_8b_5d"])
def test_layers_metadata_equals_the_reference_identity(key):
    case, caches = cpu_caches(key)
    plane = register(caches)
    assert plane.layers == case["layers"]
    assert plane.block_bytes == case["block_bytes"]
    assert list(plane.caches) == [layer["name"] for layer in case["layers"]]


@pytest.mark.parametrize("key", ["vllm031", "qwen3_8b_5d"])
def test_span_plan_and_crc_combination_rule(key):
    """kvsnap_dp_plan's offsets and shifts, and the kernels' rule: CRC32C(block) =
    ~0 ^ ~0*x^(8L) ^ XOR_s raw(span_s) * x^(8 * bytes after span s)."""
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import _dp, _load
    case, storages, layout = golden_case(key)
    lib = _dp(_load())
    spans = (_abi.Span * len(layout.spans))()
    for dst, src in zip(spans, layout.spans):
        dst.bytes = src.bytes
    total = C.c_uint64()
    assert lib.kvsnap_dp_plan(spans, len(spans), C.byref(total)) == 0
    assert total.value == layout.block_bytes
    for dst, src in zip(spans, layout.spans):
        assert dst.offset == src.offset
        assert dst.crc_shift == oracle.xpow8n(layout.block_bytes - src.offset - src.bytes)
    packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
    init = 0xFFFFFFFF ^ oracle.gf_mulmod(0xFFFFFFFF, oracle.xpow8n(layout.block_bytes))
    for block, (_, expected) in zip(packed, case["digests"]):
        acc = 0
        for span, plan in zip(layout.spans, spans):
            raw = ~oracle.crc32c(block[span.offset:span.offset + span.bytes].tobytes(), 0xFFFFFFFF) & 0xFFFFFFFF
            acc ^= oracle.gf_mulmod(raw, plan.crc_shift)
        assert acc ^ init == expected


def test_lane_partials_recombine_like_the_kernels():
    """A warp's lanes each CRC the 16-byte vectors they load (lane j: bytes 16j + 512t),
    and recombine with x^(8*16*(31-j)): the coalesced kernels' arithmetic, checked on the CPU."""
    data = np.frombuffer(bytes(range(256)) * 64, dtype=np.uint8)       # 16 KiB = 32 steps of 512 bytes
    lane_regs = []
    for j in range(32):
        reg = 0
        for t in range(len(data) // 512):
            vec = data[512 * t + 16 * j:512 * t + 16 * j + 16].tobytes()
            raw = ~oracle.crc32c(vec, 0xFFFFFFFF) & 0xFFFFFFFF
            reg = oracle.gf_mulmod(reg, oracle.xpow8n(512)) ^ raw
        lane_regs.append(reg)
    total = 0
    for j, reg in enumerate(lane_regs):
        total ^= oracle.gf_mulmod(reg, oracle.xpow8n(16 * (31 - j)))
    init = 0xFFFFFFFF ^ oracle.gf_mulmod(0xFFFFFFFF, oracle.xpow8n(len(data)))
    assert total ^ init == oracle.crc32c(data.tobytes())


@pytest.mark.parametrize("seg,length", [(1024, 4096), (2048, 8192), (1024, 4096 - 640)])
def test_segment_lanes_recombine_like_the_hbm_kernels(seg, length):
    """The device-memory kernels' arithmetic, checked on the CPU: a unit front-padded to 4 segments
    of `seg` bytes; lane (r, s) folds 16-byte slot s of every 128-byte line of segment r into four
    chains (word k, then the 124 bytes to the same word of the next line); Horner over the chains
    with x^32, the lane's factor x^(8 * (16 * (7 - s) + seg * (3 - r))), and the XOR over lanes give
    raw(unit) * x^(8 * 124), the factor the finish step divides out."""
    rng = np.random.default_rng(seg + length)
    unit = rng.integers(0, 256, length, dtype=np.uint8).tobytes()
    padded = bytes(4 * seg - length) + unit
    line_step, x32 = oracle.xpow8n(128), oracle.xpow8n(4)
    total = 0
    for lane in range(32):
        r, s = lane >> 3, lane & 7
        chains = [0, 0, 0, 0]
        for line in range(seg // 128):
            at = r * seg + line * 128 + 16 * s
            for k in range(4):
                word = int.from_bytes(padded[at + 4 * k:at + 4 * k + 4], "little")
                chains[k] = oracle.gf_mulmod(chains[k] ^ word, line_step)
        h = oracle.gf_mulmod(oracle.gf_mulmod(oracle.gf_mulmod(chains[0], x32) ^ chains[1], x32) ^ chains[2], x32)
        h ^= chains[3]
        total ^= oracle.gf_mulmod(h, oracle.xpow8n(16 * (7 - s) + seg * (3 - r)))
    raw = ~oracle.crc32c(unit, 0xFFFFFFFF) & 0xFFFFFFFF
    assert total == oracle.gf_mulmod(raw, oracle.xpow8n(124))


def test_hbm_flags_by_model_shape():
    """The unit cut the plane asks the device-memory kernels for, by registered span sizes."""
    from kvsnap_b200 import _abi
    HBM, RUNS, PAIRS, SPLIT2, SPLIT4 = _abi.HBM, _abi.RUNS, _abi.PAIRS, _abi.SPLIT2, _abi.SPLIT4
    cases = [
        ([32 << 10] * 72, HBM | SPLIT2),            # Qwen3-8B: 36 layers x K, V of 8 heads
        ([64 << 10] * 128, HBM | SPLIT4),           # 16 KV heads a rank
        ([16 << 10] * 128, HBM),                    # Qwen3-32B TP-2 shard
        ([8 << 10] * 128, HBM | RUNS),              # TP-4 shard
        ([4 << 10] * 128, HBM | RUNS | PAIRS),      # TP-8 shard
        ([2 << 10] * 6, HBM | RUNS | PAIRS),
        ([4 << 10] * 3, HBM | RUNS),                # an odd count does not pair
        ([4 << 10, 8 << 10], HBM | RUNS),           # sizes differ: runs only
        ([34816] * 4, HBM),                         # 32 KiB + 2 KiB: no 16 KiB pieces
        ([32 << 10, 16 << 10], HBM),
    ]
    for spans, want in cases:
        assert _abi.hbm_flags(spans, 16) == want, (spans[:2], len(spans))
        assert _abi.hbm_flags(spans, 8) == 0


def test_runs_coalesce_like_the_reference_copy_count():
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    size = 100
    a, b = object(), object()
    for chunk_blocks in (1, 2, 3, 64):
        targets = [(a, 0), (a, 100), (a, 200), (b, 0), (a, 300), (a, 400), (b, 100), (b, 200)]
        ours = 0
        per = max(1, min(len(targets), chunk_blocks))
        for first in range(0, len(targets), per):
            ours += len(list(TorchBlockDataPlane._runs(targets, first, min(len(targets), first + per), size)))
        keyed = [(id(x), o) for x, o in targets]
        assert ours == oracle.save_copy_count(keyed, size, chunk_blocks * size)


@pytest.mark.parametrize("spans, n, slot", [([32768] * 72, 512, 128 << 20), ([4096] * 128, 2048, 128 << 20),
                                            ([32768] * 72, 8192, 128 << 20), ([8192, 8192, 48, 16, 4096] * 3, 9, 4096),
                                            ([1 << 20] * 4, 64, 1 << 20), ([16] * 40, 3, 64)])
def test_column_plan_covers_every_block_byte_in_sha_chunks(spans, n, slot):
    """The staged save's column plan: consecutive spans, whole 64-byte chunks before the last column,
    every byte once, and a slot's group of columns within the slot unless a single column is larger."""
    from kvsnap_b200.dataplane import column_plan
    group, stride, columns = column_plan(spans, n, slot)
    assert columns[0][0] == 0 and columns[-1][1] == len(spans)
    offset = 0
    for (s0, s1, at, nbytes), nxt in zip(columns, columns[1:] + [None]):
        assert s1 > s0 and at == offset and nbytes == sum(spans[s0:s1])
        offset += nbytes
        if nxt is not None:
            assert nxt[0] == s1 and offset % 64 == 0
    assert offset == sum(spans)
    assert stride % 16 == 0 and stride >= max(c[3] for c in columns)
    assert 1 <= group <= n
    assert group * stride <= slot or group == 1


def test_even_pitch_finds_one_spacing_or_none():
    """A bounded save lands a group's column by one copy-engine transfer only when one pitch, at least
    a block, spaces all its targets."""
    from kvsnap_b200.dataplane import _even_pitch
    size = 4096
    assert _even_pitch([1000], 0, 1, size) == size
    assert _even_pitch([0, 4096, 8192, 12288], 0, 4, size) == 4096
    assert _even_pitch([0, 4112, 8224, 12336], 1, 4, size) == 4112
    assert _even_pitch([0, 4096, 8192, 12300], 0, 4, size) is None       # the last gap differs
    assert _even_pitch([0, 2048, 4096], 0, 3, size) is None                # targets would overlap
    assert _even_pitch([8192, 4096, 0], 0, 3, size) is None                # descending addresses
    assert _even_pitch([5, 0, 4096, 8192, 1], 1, 4, size) == 4096          # only the group's range counts
