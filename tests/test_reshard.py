"""Tensor-parallel regroup: a TP-(T*g) snapshot restored at TP-T.

No reference code exists (the reference misses on a TP-size change), so parity
is defined by slicing the full-head KV (oracle.slice_heads): after the regroup
rank r's cache blocks must equal the TP-T slice of the saved blocks, and
re-saving them must give the packed bytes, CRC32C and SHA-256 a TP-T save of
the same KV gives. CPU tests cover the plan, the shard layout and the rank
exchange over gloo; GPU tests run the kernel in one process and the whole
collective in two processes (gloo for the plumbing, CUDA IPC for the shards).
"""
import ctypes as C
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import kvgen
from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]
LAYERS, BLOCKS, HEADS, DIM = 3, 12, 8, 128


def full_kv(seed=5):
    """Per layer a full-head [2, B, 16, H, D] bf16 array (as uint16 bits)."""
    return {f"model.layers.{i}": kvgen.random_bytes(seed * 100 + i, 2 * BLOCKS * 16 * HEADS * DIM * 2)
            .view(np.uint16).reshape(2, BLOCKS, 16, HEADS, DIM) for i in range(LAYERS)}


def sliced_layout(full, tp, rank):
    """Oracle storages and layout of rank ``rank``'s shard at TP size ``tp``."""
    storages, views = {}, {}
    for name, kv in full.items():
        part = oracle.slice_heads(kv, tp, rank)
        storages[name] = np.ascontiguousarray(part).view(np.uint8).reshape(-1)
        views.update(oracle.split_5d(name, name, 0, BLOCKS, 16, HEADS // tp, DIM, 2))
    return storages, oracle.register(views, 16)


# ---- CPU: plan, shard layout, exchange ------------------------------------------------------------------

def test_plan_maps_shards_to_destinations():
    from kvsnap_b200.reshard import RegroupPlan
    plan = RegroupPlan(8, 4)
    assert plan.groups == 2
    assert [plan.sources(r) for r in range(4)] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert [plan.destination(s) for s in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]
    with pytest.raises(ValueError):
        RegroupPlan(6, 4)
    with pytest.raises(ValueError):
        plan.sources(4)


@pytest.mark.parametrize("src_tp,dst_tp", [(8, 4), (8, 2), (2, 1), (8, 1)])
def test_shard_layout_is_the_smaller_tp_slice_layout(src_tp, dst_tp):
    """The shard spans derived from a TP-dst registration equal the oracle layout of a TP-src slice."""
    from kvsnap_b200 import _abi
    from kvsnap_b200.reshard import shard_spans
    full = full_kv()
    _, dst = sliced_layout(full, dst_tp, 0)
    _, src = sliced_layout(full, src_tp, 0)
    spans = (_abi.Span * len(dst.spans))()
    for o, s in zip(spans, dst.spans):
        o.bytes, o.tokens, o.row_bytes = s.bytes, 16, DIM * 2
        o.token_pitch = s.stride[1] * s.elem
    out, total = shard_spans(spans, src_tp // dst_tp)
    assert total == src.block_bytes
    for o, s in zip(out, src.spans):
        assert (o.offset, o.bytes, o.token_pitch) == (s.offset, s.bytes, s.stride[1] * s.elem)


def test_regroup_by_slicing_equals_the_destination_slice():
    full = full_kv()
    for r in range(4):
        joined = {n: np.concatenate([oracle.slice_heads(kv, 8, 2 * r), oracle.slice_heads(kv, 8, 2 * r + 1)], 3)
                  for n, kv in full.items()}
        assert all(np.array_equal(joined[n], oracle.slice_heads(full[n], 4, r)) for n in full)


def _exchange_worker(rank, world, port, results):
    import torch.distributed as dist
    from kvsnap_b200.reshard import exchange
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        failure = "shard of rank 1 failed its CRC32C check" if rank == 1 else None
        failures, everyone = exchange((f"handle-{rank}".encode(), failure))
        results[rank] = (failures, [h for h, _ in everyone])
    finally:
        dist.destroy_process_group()


def test_a_failed_shard_reaches_every_rank_over_gloo():
    import torch.multiprocessing as mp
    port = 29500 + os.getpid() % 1000
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.start_processes(_exchange_worker, args=(2, port, results), nprocs=2, start_method="spawn")
        for rank in range(2):
            failures, handles = results[rank]
            assert failures == ["shard of rank 1 failed its CRC32C check"]
            assert handles == [b"handle-0", b"handle-1"]


# ---- GPU ------------------------------------------------------------------------------------------------

def _cuda_caches(storages, heads):
    return {name: torch.from_numpy(buf.copy()).cuda().view(torch.bfloat16).view(2, BLOCKS, 16, heads, DIM)
            for name, buf in storages.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("src_tp,dst_tp,rank", [(8, 4, 0), (8, 4, 3), (8, 2, 1), (2, 1, 0)])
def test_regroup_kernel_rebuilds_the_destination_shard(src_tp, dst_tp, rank):
    from kvsnap_b200.dataplane import TorchBlockDataPlane, _dp
    from kvsnap_b200.reshard import RegroupPlan, shard_spans
    from kvsnap_b200 import _abi
    full = full_kv()
    plan = RegroupPlan(src_tp, dst_tp)
    saved, restored = kvgen.disjoint_block_sets(3, BLOCKS, 4)
    dst_storages, dst_layout = sliced_layout(full, dst_tp, rank)
    zeros = {n: np.zeros_like(b) for n, b in dst_storages.items()}
    caches = _cuda_caches(zeros, HEADS // dst_tp)
    plane = TorchBlockDataPlane(caches, 16, 64 << 20)
    plane.warm_up()
    try:
        lib = _dp(plane.pool.lib)
        shards = []
        for src in plan.sources(rank):
            storages, layout = sliced_layout(full, src_tp, src)
            packed = oracle.pack(storages, layout, saved, len(saved) * 16)
            shards.append(torch.from_numpy(np.concatenate(packed)).cuda())
            shard_bytes = layout.block_bytes
        dst_host = (_abi.Span * len(plane.layers)).from_buffer_copy(plane._span_table.cpu().numpy().tobytes())
        src_spans, total = shard_spans(dst_host, plan.groups)
        assert total == shard_bytes
        src_table = torch.frombuffer(bytearray(bytes(src_spans)), dtype=torch.uint8).cuda()
        rows = [shards[q].data_ptr() + i * shard_bytes for i in range(len(saved)) for q in range(plan.groups)]
        table = torch.tensor(rows + restored, dtype=torch.int64, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert lib.kvsnap_dp_regroup(plane._span_table.data_ptr(), src_table.data_ptr(), len(plane.layers),
                                     table.data_ptr(), plan.groups, table[len(rows):].data_ptr(), len(saved),
                                     status.data_ptr(), 0, torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        # The cache now holds the destination slice of the saved blocks, and nothing else changed.
        for name, tensor in caches.items():
            got = tensor.view(torch.int16).cpu().numpy().view(np.uint16)
            want = oracle.slice_heads(full[name], dst_tp, rank)
            expect = np.zeros_like(want)
            expect[:, restored] = want[:, saved]
            assert np.array_equal(got, expect), name
        # Re-saving gives the bytes and digests of a save at the destination size.
        targets = [plane.pool.reserve(plane.block_bytes) for _ in restored]
        digests = []
        plane.save_gather(restored, [(a, 0) for a in targets], len(restored) * 16, digests=digests)
        reference = oracle.pack(dst_storages, dst_layout, saved, len(saved) * 16)
        assert [a.read_range(0, plane.block_bytes) for a in targets] == [b.tobytes() for b in reference]
        assert [tuple(d) for d in digests] == oracle.digests(reference)
    finally:
        plane.close()


def _collective_worker(rank, world, port, env):
    os.environ.update(env)
    sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
    import torch.distributed as dist
    from kvsnap_b200.dataplane import CorruptBlockError, TorchBlockDataPlane
    from kvsnap_b200.reshard import Regrouper, RegroupPlan, regroup_restore
    device = rank % torch.cuda.device_count()
    torch.cuda.set_device(device)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        full = full_kv()
        plan = RegroupPlan(world, 1)
        saved, restored = kvgen.disjoint_block_sets(4, BLOCKS, 5)
        dst_storages, dst_layout = sliced_layout(full, 1, 0)
        caches = _cuda_caches({n: np.zeros_like(b) for n, b in dst_storages.items()}, HEADS)
        plane = TorchBlockDataPlane(caches, 16, 64 << 20)
        storages, layout = sliced_layout(full, world, rank)
        packed = oracle.pack(storages, layout, saved, len(saved) * 16)
        crcs = [oracle.crc32c(b) for b in packed]
        snapshot = plane.pool.reserve(layout.block_bytes * len(saved))
        for i, block in enumerate(packed):
            C.memmove(snapshot.pointer + i * layout.block_bytes, block.ctypes.data, layout.block_bytes)
        sources = [(snapshot, i * layout.block_bytes) for i in range(len(saved))]
        # A corrupt shard on the last rank fails the restore on every rank, before any cache write.
        bad = list(crcs)
        if rank == world - 1:
            bad[2] ^= 1
        with_error = None
        try:
            regroup_restore(plane, plan, rank, restored, sources, expected_crc32c=bad)
        except CorruptBlockError as exc:
            with_error = str(exc)
        assert with_error and "failed its CRC32C check" in with_error
        for name, tensor in caches.items():
            assert not tensor.view(torch.int16).any().item(), "cache written despite a corrupt shard"
        launches = regroup_restore(plane, plan, rank, restored, sources, expected_crc32c=crcs)
        assert launches == (1 if rank == 0 else 0)

        def check(into, count):
            if rank == 0:
                for name, tensor in caches.items():
                    got = tensor.view(torch.int16).cpu().numpy().view(np.uint16)
                    expect = np.zeros_like(full[name])
                    expect[:, into[:count]] = full[name][:, saved[:count]]
                    assert np.array_equal(got, expect), name

        check(restored, len(saved))
        # A kept Regrouper: a smaller restore, a corrupt one, then a larger one that grows
        # every source buffer (so every destination remaps), all through the same object.
        for tensor in caches.values():
            tensor.zero_()
        regrouper = Regrouper(plane, plan, rank)
        try:
            assert regrouper.restore(restored[:2], sources[:2], expected_crc32c=crcs[:2]) == (1 if rank == 0 else 0)
            check(restored, 2)
            with_error = None
            try:
                regrouper.restore(restored, sources, expected_crc32c=bad)
            except CorruptBlockError as exc:
                with_error = str(exc)
            assert with_error and "failed its CRC32C check" in with_error
            check(restored, 2)
            regrouper.restore(restored, sources, expected_crc32c=crcs)
            check(restored, len(saved))
        finally:
            regrouper.close()
        dist.barrier()
        snapshot.close()
        plane.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_process_regroup_over_ipc():
    """Two ranks (two GPUs when present, else both on one): rank 0 restores at TP-1 from the
    TP-2 shards of both ranks, rank 1's read through CUDA IPC."""
    import torch.multiprocessing as mp
    port = 29600 + os.getpid() % 1000
    env = {"PYTHONPATH": os.pathsep.join([str(ROOT), str(ROOT / "tests")]), "NCCL_NVLS_ENABLE": "0"}
    mp.start_processes(_collective_worker, args=(2, port, env), nprocs=2, start_method="spawn")
