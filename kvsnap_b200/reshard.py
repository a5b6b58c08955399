"""Restore a tensor-parallel snapshot at a smaller TP size: regroup KV-head shards over NVLink.

The reference restores a snapshot only at the TP size it was saved at; any
other size is a miss (kvsnap/connector/vllm.py:9-14, models.py ``rank_segments``).
This module adds the TP-8 -> TP-4 case (any T*g -> T): rank r of the smaller
group holds heads [r*H, (r+1)*H) of every layer, which the larger group saved
as g shards, source ranks r*g .. r*g+g-1, each with H/g heads.

Design (one process per GPU, torch.distributed for the plumbing):

1. every source rank copies its own shard's packed blocks from pinned host
   memory into device memory it can share (``kvsnap_dp_device_alloc``) and, if
   CRCs are given, checks them there on the GPU;
2. the ranks exchange CUDA IPC handles (``all_gather_object``) and each
   destination rank maps its g source buffers (``kvsnap_dp_ipc_open``; its own
   buffer is used directly);
3. a barrier orders step 1 before the reads; the destination rank's
   ``kvsnap_dp_regroup`` kernel reads the shards with plain loads, peers over
   NVLink, and writes each (head, token) row into its own cache blocks;
4. a second barrier keeps the source buffers alive until every reader is done.

``Regrouper`` keeps the shard buffer, its handle and the peer mappings from
one restore to the next; ``regroup_restore`` is the one-shot form.

Parity is defined by slicing: after the regroup, rank r's cache blocks hold
exactly the heads a TP-size-T save of the same KV would hold
(oracle ``slice_heads``), and re-saving them gives the same packed bytes, CRCs
and content ids as the reference's save at that size.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

from . import _abi


@dataclass(frozen=True)
class RegroupPlan:
    """Which source ranks feed which destination rank, for TP ``src_tp`` -> ``dst_tp``."""
    src_tp: int
    dst_tp: int

    def __post_init__(self):
        if self.src_tp <= 0 or self.dst_tp <= 0 or self.src_tp % self.dst_tp:
            raise ValueError("the source TP size must be a multiple of the destination TP size")

    @property
    def groups(self) -> int:
        return self.src_tp // self.dst_tp

    def sources(self, dst_rank: int) -> list:
        """Source shard ranks of destination rank ``dst_rank``, in head order."""
        if not 0 <= dst_rank < self.dst_tp:
            raise ValueError("destination rank out of range")
        return [dst_rank * self.groups + q for q in range(self.groups)]

    def destination(self, src_rank: int) -> int:
        if not 0 <= src_rank < self.src_tp:
            raise ValueError("source rank out of range")
        return src_rank // self.groups


def shard_spans(dst_spans, groups: int):
    """One source shard's packed layout from this rank's registered spans.

    Same spans in the same (layer-name) order, each with ``heads / groups``
    heads: bytes divide by ``groups``; a token-major span (token slots more than
    one row apart) also has its token pitch divided. Offsets and CRC shifts are
    then planned as for any packed block.
    """
    from .dataplane import _dp, _load
    out = (_abi.Span * len(dst_spans))()
    for o, d in zip(out, dst_spans):
        if d.bytes % groups or (d.bytes // (d.tokens * d.row_bytes)) % groups:
            raise ValueError("heads per layer must divide by the TP ratio")
        o.bytes = d.bytes // groups
        o.tokens, o.row_bytes = d.tokens, d.row_bytes
        o.token_pitch = d.token_pitch if d.token_pitch == d.row_bytes else d.token_pitch // groups
        o.nblocks = 0
    lib = _dp(_load())
    total = C.c_uint64()
    if lib.kvsnap_dp_plan(out, len(out), C.byref(total)) < 0:
        raise RuntimeError(lib.kvsnap_cuda_error().decode())
    return out, total.value


class SharedBuffer:
    """Device memory another process on the box can map (CUDA IPC)."""

    def __init__(self, lib, size: int, device: int):
        self.lib, self.size, self.device = lib, size, device
        ptr = C.c_void_p()
        if lib.kvsnap_dp_device_alloc(size, device, C.byref(ptr)) < 0:
            raise RuntimeError(lib.kvsnap_cuda_error().decode())
        self.ptr = ptr.value

    def handle(self) -> bytes:
        out = C.create_string_buffer(64)
        if self.lib.kvsnap_dp_ipc_export(self.ptr, out) < 0:
            raise RuntimeError(self.lib.kvsnap_cuda_error().decode())
        return out.raw

    def close(self):
        if self.ptr:
            self.lib.kvsnap_dp_device_free(self.ptr)
            self.ptr = 0


def open_peer(lib, handle: bytes, device: int) -> int:
    ptr = C.c_void_p()
    if lib.kvsnap_dp_ipc_open(handle, device, C.byref(ptr)) < 0:
        raise RuntimeError(lib.kvsnap_cuda_error().decode())
    return ptr.value


def close_peer(lib, ptr: int) -> None:
    if lib.kvsnap_dp_ipc_close(ptr) < 0:
        raise RuntimeError(lib.kvsnap_cuda_error().decode())


class Regrouper:
    """A TP regroup that keeps its shard buffer and peer mappings from one restore to the next.

    Collective: every rank of ``group`` builds one, calls ``restore`` the same
    number of times and then ``close``. Source rank s of the plan runs on
    torch.distributed rank s; destination rank r on rank r.

    What a one-shot regroup pays on every call is paid here once:
    - the shareable device buffer of this rank's shard, kept and grown on demand;
    - its CUDA IPC handle, exported once per buffer;
    - the destination's mappings of its peers' buffers, reopened only when a
      peer's handle changes.
    A buffer replaced by a larger one stays alive until the barrier that ends
    the restore, by which time every destination has closed its mapping.
    """

    def __init__(self, plane, plan: RegroupPlan, rank: int, *, group=None, is_destination=None):
        import torch
        from .dataplane import _dp
        self.plane, self.plan, self.rank, self.group = plane, plan, rank, group
        self.lib = _dp(plane.pool.lib)
        self.device = plane._device()
        plane._spans()
        self.stream = plane._scatter_targets()
        host_spans = _abi.Span * len(plane.layers)
        dst_host = host_spans.from_buffer_copy(plane._span_table.cpu().numpy().tobytes())
        self.src_spans, self.shard_bytes = shard_spans(dst_host, plan.groups)
        self.src_table = torch.frombuffer(bytearray(bytes(self.src_spans)), dtype=torch.uint8).to(self.device)
        self.is_source = rank < plan.src_tp
        self.is_destination = rank < plan.dst_tp if is_destination is None else is_destination
        self.buffer, self.handle, self.retired = None, None, []
        self.peers = {}                  # source rank -> (IPC handle, mapped pointer)
        self.closed = False

    def restore(self, block_ids, shard_sources, *, expected_crc32c=None, timings=None) -> int:
        """Regroup one snapshot into this rank's cache blocks; returns the launches on this rank.

        ``shard_sources``: this rank's own shard of the snapshot,
        ``[(allocation, offset), ...]`` one packed block per entry of ``block_ids``
        (source ranks only; ``None`` elsewhere). ``block_ids``: the destination
        rank's cache blocks (ignored on ranks that are not a destination).
        ``expected_crc32c``: this rank's shard CRCs, checked on the GPU before
        anyone reads the shard; a mismatch on any rank raises CorruptBlockError on
        every rank with no cache written. ``timings``: receives the host-side
        seconds of the stage, exchange and regroup phases and the regroup
        kernel's device milliseconds.
        """
        import time
        import torch
        import torch.distributed as dist
        from .dataplane import CorruptBlockError
        if self.closed:
            raise RuntimeError("regrouper is closed")
        n = len(block_ids)
        # 1. Source ranks stage their shard in shareable device memory and check it.
        #    A failure here is carried into the exchange, so every rank still takes
        #    the same collective steps and all of them raise it afterwards.
        failure = None
        t0 = time.perf_counter()
        try:
            if self.is_source and n:
                self._stage(n, shard_sources, expected_crc32c)
        except CorruptBlockError as exc:
            failure = str(exc)
        except Exception as exc:          # noqa: BLE001 - reported to every rank, then raised
            failure = f"rank {self.rank}: {type(exc).__name__}: {exc}"

        # 2. Exchange handles and verdicts; every rank takes the same collective steps.
        t1 = time.perf_counter()
        failures, everyone = exchange((self.handle if self.is_source else None, failure), self.group)
        t2 = time.perf_counter()
        launches = 0
        try:
            if self.is_destination and n:
                # Remap every changed peer now, failed restore or not, so that no
                # mapping of a buffer its owner retires outlives the barrier below.
                for src in self.plan.sources(self.rank):
                    if src != self.rank and everyone[src][0] is not None:
                        self._shard(src, everyone[src][0])
            if not failures and self.is_destination and n:
                shards = [self._shard(src, everyone[src][0]) for src in self.plan.sources(self.rank)]
                rows = [shards[q] + i * self.shard_bytes for i in range(n) for q in range(self.plan.groups)]
                device, stream = self.device, self.stream
                with torch.cuda.stream(stream):
                    table = torch.tensor(rows + list(block_ids), dtype=torch.int64, device=device)
                    status = torch.zeros(1, dtype=torch.int32, device=device)
                    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    begin.record(stream)
                    if self.lib.kvsnap_dp_regroup(self.plane._span_table.data_ptr(), self.src_table.data_ptr(),
                                                  len(self.plane.layers), table.data_ptr(), self.plan.groups,
                                                  table[len(rows):].data_ptr(), n, status.data_ptr(), 0,
                                                  stream.cuda_stream) < 0:
                        raise RuntimeError(self.lib.kvsnap_cuda_error().decode())
                    end.record(stream)
                    launches = 1
                stream.synchronize()
                if timings is not None:
                    timings["kernel_ms"] = begin.elapsed_time(end)
                if int(status.item()):
                    raise RuntimeError(f"regroup kernel reported status {int(status.item())}")
        finally:
            # 3. Nobody frees a shard another rank may still be reading.
            dist.barrier(group=self.group)
            if timings is not None:
                timings.update(stage_s=t1 - t0, exchange_s=t2 - t1, regroup_s=time.perf_counter() - t2)
            for old in self.retired:
                old.close()
            self.retired = []
        if failures:
            raise CorruptBlockError("; ".join(failures))
        return launches

    def close(self):
        """Collective: close the peer mappings, wait for every rank, then free this rank's buffer."""
        import torch.distributed as dist
        if self.closed:
            return
        self.closed = True
        try:
            for _, ptr in self.peers.values():
                close_peer(self.lib, ptr)
            self.peers = {}
        finally:
            dist.barrier(group=self.group)
            for buf in [self.buffer, *self.retired]:
                if buf is not None:
                    buf.close()
            self.buffer, self.handle, self.retired = None, None, []

    def _shard(self, src: int, handle) -> int:
        """Device address of source rank ``src``'s shard: this rank's own buffer, or a peer mapping."""
        if src == self.rank:
            return self.buffer.ptr
        if handle is None:
            raise RuntimeError(f"source rank {src} shared no shard")
        cached = self.peers.get(src)
        if cached is not None and cached[0] == handle:
            return cached[1]
        if cached is not None:
            del self.peers[src]
            close_peer(self.lib, cached[1])
        ptr = open_peer(self.lib, handle, self.device.index)
        self.peers[src] = (handle, ptr)
        return ptr

    def _stage(self, n, shard_sources, expected_crc32c):
        """Copy this rank's shard into its shareable buffer (grown if needed) and check its CRCs there."""
        need = n * self.shard_bytes
        if self.buffer is None or self.buffer.size < need:
            if self.buffer is not None:
                self.retired.append(self.buffer)
            self.buffer, self.handle = None, None
            self.buffer = SharedBuffer(self.lib, need, self.device.index)
            self.handle = self.buffer.handle()
        _stage_shard(self.lib, self.plane, self.stream, self.rank, n, self.shard_bytes, shard_sources,
                     expected_crc32c, self.buffer)


def regroup_restore(plane, plan: RegroupPlan, rank: int, block_ids, shard_sources, *, group=None,
                    expected_crc32c=None, is_destination=None, timings=None):
    """One collective TP regroup restore; every rank of ``group`` calls it.

    ``plane``: this rank's TorchBlockDataPlane, registered at the destination TP
    size (its caches hold this rank's heads). The other arguments are those of
    ``Regrouper.restore``. A caller that regroups repeatedly keeps a Regrouper
    instead, which skips the per-call buffer and IPC setup.
    """
    regrouper = Regrouper(plane, plan, rank, group=group, is_destination=is_destination)
    try:
        return regrouper.restore(block_ids, shard_sources, expected_crc32c=expected_crc32c, timings=timings)
    finally:
        regrouper.close()


def exchange(mine, group=None):
    """All-gather every rank's (IPC handle, failure); returns (failures, all entries)."""
    import torch.distributed as dist
    everyone = [None] * dist.get_world_size(group)
    dist.all_gather_object(everyone, mine, group=group)
    return [f for _, f in everyone if f], everyone


def _stage_shard(lib, plane, stream, rank, n, shard_bytes, shard_sources, expected_crc32c, buffer):
    """Copy this rank's shard into ``buffer`` and check its CRCs there.

    Runs of sources adjacent in one allocation move in one copy.
    """
    import torch
    from .dataplane import CorruptBlockError
    if shard_sources is None or len(shard_sources) != n:
        raise ValueError("one shard block per restored block is required")
    for allocation, offset in shard_sources:
        allocation._open()
        if offset < 0 or offset + shard_bytes > allocation.size:
            raise ValueError("shard source outside its allocation")
    device = plane._device()
    try:
        with torch.cuda.stream(stream):
            i = 0
            while i < n:
                allocation, offset = shard_sources[i]
                j = i + 1
                while j < n and shard_sources[j][0] is allocation and \
                        shard_sources[j][1] == offset + (j - i) * shard_bytes:
                    j += 1
                allocation.copy(buffer.ptr + i * shard_bytes, (j - i) * shard_bytes, offset, to_host=False)
                i = j
            if expected_crc32c is not None:
                table = torch.tensor([buffer.ptr + i * shard_bytes for i in range(n)], dtype=torch.int64,
                                     device=device)
                crc = torch.empty(n, dtype=torch.int32, device=device)
                status = torch.zeros(1, dtype=torch.int32, device=device)
                expect = torch.tensor([v - (1 << 32) if v >= 1 << 31 else v for v in expected_crc32c],
                                      dtype=torch.int32, device=device)
                vec = (16 | _abi.HBM) if shard_bytes % 16 == 0 else 8
                if lib.kvsnap_dp_crc32c(table.data_ptr(), n, shard_bytes, crc.data_ptr(), expect.data_ptr(),
                                        status.data_ptr(), vec, 0, stream.cuda_stream) < 0:
                    raise RuntimeError(lib.kvsnap_cuda_error().decode())
                if int(status.item()) & _abi.CRC_MISMATCH:
                    raise CorruptBlockError(f"shard of rank {rank} failed its CRC32C check")
        stream.synchronize()
    except BaseException:
        stream.synchronize()
        raise
