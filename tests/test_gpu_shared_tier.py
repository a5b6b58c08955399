"""The cross-owner host tier on a B200: one worker restores a snapshot another worker's pinned pool holds.

The owner (this process) saves a session with ``save_gather`` into per-block
allocations of a shared pinned pool, its content ids and CRCs from the GPU,
and hands out the blocks' locations. A second worker process on the same GPU
maps the owner's pool read-only (kvsnap_b200.sharedtier) and restores the
blocks in place into its own cache with ``expected_crc32c``: every restored
span equals the oracle's packed bytes, and a wrong CRC is refused before any
write. The reference moves the same bytes over a Unix socket and a host copy
(kvsnap/connector/vllm.py:524-534, connector/volatile.py:87-138).
"""
import json
import subprocess
import sys
from pathlib import Path

import pytest

from test_gpu_full_size import FormulaCache, release

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

WORKER = r"""
import json, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/tests"]
import torch
from oracle import oracle
from test_gpu_full_size import FormulaCache, release
from kvsnap_b200.dataplane import CorruptBlockError, TorchBlockDataPlane
from kvsnap_b200.sharedtier import SharedBlocks
job = json.loads(sys.argv[2])
cache = FormulaCache(job["restore_seed"], job["layers"], job["pool"], 8)
plane = TorchBlockDataPlane(cache.caches, 16, 64 << 20)
plane.warm_up()
view = SharedBlocks(job["segment"], 0)
sources = view.sources(job["locations"])
ids = torch.tensor(job["restored"], device="cuda")
before = {k: t.view(torch.int16)[:, ids].clone() for k, t in cache.caches.items()}
bad = list(job["crcs"])
bad[3] ^= 1
try:
    plane.load_scatter(job["restored"], sources, expected_crc32c=bad)
    rejected = False
except CorruptBlockError as err:
    rejected = err.blocks == [3]
untouched = all(torch.equal(t.view(torch.int16)[:, ids], before[k]) for k, t in cache.caches.items())
plane.load_scatter(job["restored"], sources, expected_crc32c=job["crcs"])
# What the owner packed: the oracle's bytes of its own cache.
owner = FormulaCache(job["save_seed"], job["layers"], job["pool"], 8)
packed = oracle.pack(owner.storages, owner.layout, job["saved"], job["tokens"])
rows = torch.from_numpy(__import__("numpy").stack(packed)).cuda()
exact = all(torch.equal(cache.rows(cache.raw, span)[ids], rows[:, span.offset:span.offset + span.bytes])
            for span in cache.layout.spans)
view.close()
release(plane, cache)
print(json.dumps({"rejected": rejected, "untouched": untouched, "exact": exact}), flush=True)
"""


def test_a_second_worker_restores_the_owners_blocks_in_place():
    import random
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    from kvsnap_b200.sharedtier import locations, new_segment_name
    layers, pool_blocks, n = 12, 600, 48
    cache = FormulaCache(51, layers, pool_blocks, 8)
    size = cache.layout.block_bytes
    plane = TorchBlockDataPlane(cache.caches, 16, n * (size + 16) + (64 << 20), shared_name=new_segment_name())
    try:
        plane.warm_up()
        rng = random.Random(4)
        saved = rng.sample(range(1, pool_blocks), n)
        restored = rng.sample(range(1, pool_blocks), n)
        tokens = n * 16 - 6
        owned = [plane.pool.reserve(size) for _ in range(n)]
        digests = []
        plane.save_gather(saved, [(a, 0) for a in owned], tokens, digests=digests)
        job = {"segment": plane.pool.shared_name, "locations": locations(plane.pool, owned),
               "crcs": [c for _, c in digests], "saved": saved, "restored": restored, "tokens": tokens,
               "layers": layers, "pool": pool_blocks, "save_seed": 51, "restore_seed": 52}
        worker = subprocess.run([sys.executable, "-c", WORKER, str(ROOT), json.dumps(job)], capture_output=True,
                                text=True, timeout=600)
        assert worker.returncode == 0, worker.stderr[-3000:]
        result = json.loads(worker.stdout.strip().splitlines()[-1])
        assert result == {"rejected": True, "untouched": True, "exact": True}
        for a in owned:
            a.close()
    finally:
        release(plane, cache)
