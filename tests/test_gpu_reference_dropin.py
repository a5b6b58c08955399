"""This data plane and the reference's own, side by side on a B200 over the same KV cache.

The reference (installed under baseline/_ref with its CUDA pool) runs its
stock ``TorchBlockDataPlane``: torch ``index_select`` + ``cat`` and
``cudaMemcpyAsync`` for the save (kvsnap/connector/dataplane.py:388-437), its
Triton kernel for the restore (kvsnap/connector/copy_kernel.py:23-49). Ours
runs with the same arguments. Both must agree on the registered layers, every
packed byte (per-block and one-buffer targets, a partial last block), the
save's copy count, the restore's launch count and progress, and every byte of
the cache after the restore, for the vLLM 0.31 registration of the
reference's own GPU test (tests/connector/test_copy_kernel_cuda.py:21-66) and
for the 5-D paged layout split into its K and V views.

Then the connector's save (kvsnap/connector/vllm.py:581-624) on our plane:
the content ids and CRCs our GPU returns with ``digests=`` equal the ones the
reference's own host code computes over the same pinned blocks, both the
host tier's per-allocation ``_digest`` (connector/volatile.py:141-151) and the
durable tier's ``_prepare_payloads`` (store/store.py:616-629).
"""
import ctypes as C
import random

import numpy as np
import pytest
import torch

import kvgen
from refpath import reference

pytestmark = pytest.mark.gpu


def _vllm031(seed, layers=6, blocks=96):
    raw = torch.empty(layers * blocks * 16 * 8 * 256 * 2, dtype=torch.uint8, device="cuda")
    kvgen.fill_random(raw, seed)
    backing = raw.view(torch.bfloat16).view(layers, blocks, 16, 8, 256)
    return raw, {f"model.layers.{i}.self_attn.attn": backing[i].permute(0, 2, 1, 3) for i in range(layers)}, blocks


def _paged_split(seed, layers=12, blocks=300):
    from kvsnap_b200.dataplane import _split_paged
    raws, paged = [], {}
    for i in range(layers):
        raw = torch.empty(2 * blocks * 16 * 8 * 128 * 2, dtype=torch.uint8, device="cuda")
        kvgen.fill_random(raw, seed * 100 + i)
        raws.append(raw)
        paged[f"model.layers.{i}"] = raw.view(torch.bfloat16).view(2, blocks, 16, 8, 128)
    # The reference registers 4-D views only; both planes get the K and V views our plane registers.
    return raws, _split_paged(paged, 16), blocks


def _bits(raws):
    return [r.view(torch.int16).clone() for r in raws]


@pytest.fixture
def reference_dataplane(monkeypatch):
    dataplane = reference("connector.dataplane")
    monkeypatch.delenv("KVSNAP_CUDA_LIBRARY", raising=False)      # the reference's own pool library
    if not dataplane.resolve_cuda_library().is_file():
        pytest.skip("the reference was installed without its CUDA pool")
    return dataplane


@pytest.mark.parametrize("layout", ["vllm031", "paged-split"])
def test_reference_and_ours_pack_and_restore_the_same_bytes(reference_dataplane, layout):
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    if layout == "vllm031":
        raw, caches, blocks = _vllm031(5)
        raws = [raw]
    else:
        raws, caches, blocks = _paged_split(6)
    rng = random.Random(3)
    saved = rng.sample(range(1, blocks), 40)
    restored = rng.sample([b for b in range(1, blocks) if b not in saved], 40)
    tokens = 40 * 16 - 5
    ref = reference_dataplane.TorchBlockDataPlane(caches, 16, 256 << 20)
    ours = TorchBlockDataPlane(caches, 16, 256 << 20)
    try:
        ref.warm_up()
        ours.warm_up()
        assert ours.layers == ref.layers and ours.block_bytes == ref.block_bytes
        size, n = ours.block_bytes, len(saved)
        original = _bits(raws)
        for kind in ("one buffer", "per block"):
            packed = {}
            for name, plane in (("reference", ref), ("ours", ours)):
                if kind == "one buffer":
                    owned = [plane.pool.reserve(n * size)]
                    targets = [(owned[0], i * size) for i in range(n)]
                else:
                    owned = [plane.pool.reserve(size) for _ in range(n)]
                    targets = [(a, 0) for a in owned]
                copies = plane.save_gather(saved, targets, tokens, chunk_bytes=7 * size)
                data = b"".join(a.read_range(o, size) for a, o in targets)
                progress = []
                launches = plane.load_scatter(restored, targets, progress=progress, chunk_bytes=3 * size)
                torch.cuda.synchronize()
                packed[name] = (copies, data, launches, [left for _, left in progress], _bits(raws))
                for r, o in zip(raws, original):
                    r.view(torch.int16).copy_(o)
                for a in owned:
                    a.close()
            ref_copies, ref_data, ref_launches, ref_left, ref_after = packed["reference"]
            copies, data, launches, left, after = packed["ours"]
            assert data == ref_data, f"{kind}: packed bytes differ from the reference's"
            assert copies == ref_copies and launches == ref_launches and left == ref_left, kind
            assert all(torch.equal(a, b) for a, b in zip(after, ref_after)), f"{kind}: restored cache differs"
    finally:
        ours.close()
        ref.close()


def test_connector_save_gets_the_reference_content_ids_without_host_hashing(reference_dataplane):
    from kvsnap_b200.dataplane import PendingDigests, TorchBlockDataPlane
    volatile = reference("connector.volatile")
    store = reference("store.store")
    raws, caches, blocks = _paged_split(8)
    plane = TorchBlockDataPlane(caches, 16, 256 << 20)
    try:
        plane.warm_up()
        size = plane.block_bytes
        rng = random.Random(9)
        block_ids = rng.sample(range(1, blocks), 33)
        block_ids[20] = block_ids[3]                  # a repeated block: one blob, two segments
        tokens = 33 * 16 - 11
        # Host tier (vllm.py:589-591): one pinned allocation a block; the producer fenced first.
        owned = [plane.pool.reserve(size) for _ in block_ids]
        ready = plane.producer_event()
        ready.synchronize()
        pending = PendingDigests()
        plane.save_gather(block_ids, [(a, 0) for a in owned], tokens, digests=pending)
        gpu = [tuple(d) for d in pending.result()]
        assert gpu == [volatile._digest(a) for a in owned]
        # Durable tier (vllm.py:609-615): the blocks read back and prepared by the store.
        payloads, segments = store._prepare_payloads([a.read() for a in owned])
        assert [(s["blob_id"], s["crc32c"]) for s in segments] == gpu
        assert len(payloads) == len({g[0] for g in gpu}) == 32
        for a in owned:
            a.close()
    finally:
        plane.close()
