"""The verified restore scatter that allocates nothing (kvsnap_dp_scatter_verify_static), against the one that does.

Some callers of this data plane cannot allocate device memory: a serving worker
whose KV cache was sized to fill the GPU has no room for a CRC buffer, and host
code that must not enter an allocator that may synchronise the device cannot
call one. For them the library keeps the per-block CRC accumulators and the
verdict that gates the copy in a fixed scratch array of its own. This test
calls that entry point through the C ABI and checks, for packed blocks in
pinned host memory (the host-link kernels) and in device memory (the
segment-lane HBM kernels, with the plane's unit cut):

* on two calls in a row (the scratch keeps the previous call's contents, so
  each call must clear it) it leaves the same cache bytes and the same status
  as kvsnap_dp_scatter given a caller-allocated CRC buffer, and the oracle's;
* a bad checksum gives the same status as kvsnap_dp_scatter, but, because the
  check runs before the copy, the cache is left exactly as it was;
* a clean call after a failing one succeeds;
* a request beyond the scratch's size is refused before anything runs.

This file sorts last so that a run stopping at the first failure has already
run every other test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from cases import golden_case
from gpu_cases import cuda_5d, host_bytes
from oracle import oracle

pytestmark = pytest.mark.gpu


def _i32(values):
    return torch.tensor([v - (1 << 32) if v >= 1 << 31 else v for v in values], dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("where", ["pinned", "device"])
def test_static_scratch_scatter_matches_the_allocating_entry_point(where):
    from kvsnap_b200 import _abi
    from kvsnap_b200.dataplane import TorchBlockDataPlane, _dp
    case, storages, layout = golden_case("qwen3_8b_5d")
    _, tensors, caches = cuda_5d(case)
    plane = TorchBlockDataPlane(caches, 16, 64 << 20)
    try:
        lib = _dp(plane.pool.lib)
        spans = plane._spans()
        packed = oracle.pack(storages, layout, case["saved"], case["num_kv_tokens"])
        n, size = len(packed), plane.block_bytes
        snapshot = plane.pool.reserve(n * size)
        for i, block in enumerate(packed):
            C.memmove(snapshot.pointer + i * size, block.ctypes.data, size)
        if where == "pinned":
            base, vec = snapshot.pointer, 16
        else:
            staged = torch.empty(n * size, dtype=torch.uint8, device="cuda")
            staged.copy_(torch.from_numpy(np.concatenate(packed)))
            base, vec = staged.data_ptr(), 16 | plane._hbm
            assert vec & _abi.HBM
        sources = torch.tensor([base + i * size for i in range(n)], dtype=torch.int64, device="cuda")
        blocks = torch.tensor(case["restored"], dtype=torch.int64, device="cuda")
        good = _i32([oracle.crc32c(b) for b in packed])
        bad = _i32([oracle.crc32c(b) ^ (1 if i == 2 else 0) for i, b in enumerate(packed)])
        stream = torch.cuda.current_stream().cuda_stream
        nspans = len(plane.layers)
        originals = {name: torch.from_numpy(buf.copy()).cuda() for name, buf in storages.items()}

        def reset():
            for name, t in tensors.items():
                t.copy_(originals[name])
            torch.cuda.synchronize()

        def allocating(expect):
            reset()
            crc = torch.empty(n, dtype=torch.int32, device="cuda")
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            assert lib.kvsnap_dp_scatter(spans.data_ptr(), nspans, size, sources.data_ptr(), blocks.data_ptr(), n,
                                         crc.data_ptr(), expect.data_ptr(), 0, status.data_ptr(), vec, 0,
                                         stream) == 0
            torch.cuda.synchronize()
            return host_bytes(tensors), int(status.item())

        def static(expect):
            reset()
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            assert lib.kvsnap_dp_scatter_verify_static(spans.data_ptr(), nspans, size, sources.data_ptr(),
                                                       blocks.data_ptr(), n, expect.data_ptr(), status.data_ptr(),
                                                       vec, 0, stream) == 0
            torch.cuda.synchronize()
            return host_bytes(tensors), int(status.item())

        expected_cache = {k: v.copy() for k, v in storages.items()}
        oracle.unpack(expected_cache, layout, case["restored"], packed)
        for _ in range(2):                   # two calls in a row: the scratch must start from zero each time
            kv_a, status_a = allocating(good)
            kv_b, status_b = static(good)
            assert status_a == status_b == 0
            assert all(np.array_equal(kv_a[k], kv_b[k]) for k in kv_a)
            assert all(np.array_equal(kv_b[k], expected_cache[k]) for k in kv_b)
        for _ in range(2):
            _, status_a = allocating(bad)
            kv_b, status_b = static(bad)
            assert status_a == status_b == _abi.CRC_MISMATCH
            # Checked before the copy: the cache still holds what it held before the call.
            assert all(np.array_equal(kv_b[k], storages[k]) for k in kv_b)
        kv_b, status_b = static(good)        # a clean call after a failing one
        assert status_b == 0
        assert all(np.array_equal(kv_b[k], expected_cache[k]) for k in kv_b)

        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        too_many = _abi.STATIC_MAX_BLOCKS + 1
        assert lib.kvsnap_dp_scatter_verify_static(spans.data_ptr(), nspans, size, sources.data_ptr(),
                                                   blocks.data_ptr(), too_many, good.data_ptr(), status.data_ptr(),
                                                   vec, 0, stream) == -1
        assert "KVSNAP_DP_STATIC_MAX_BLOCKS" in lib.kvsnap_cuda_error().decode()
        snapshot.close()
    finally:
        plane.close()
