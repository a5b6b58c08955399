#!/usr/bin/env python
"""KV snapshot data-plane benchmark: 8k-token Qwen3-8B session save + restore on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark configuration 2, "Qwen3-8B shape on 1xB200"): 36 layers, each a
paged ``[2, 32768 blocks, 16 tokens, 8 kv heads, 128]`` bf16 cache filled with
seeded N(0,1) values (72 GiB of HBM), one 8192-token session = 512 blocks
(1,207,959,552 bytes packed) at seeded random block ids. One step = save the
session (gather + CRC32C + SHA-256 content ids, packed into pinned host
memory) and restore it into a disjoint set of freshly allocated blocks.

``value`` is whole-job GB/s over the GPU-timed step: saved plus restored bytes
divided by the step's device time, the block tables resident in HBM and the
kernels launched back to back (CUDA events on the data plane's streams, max
over ranks). ``e2e`` is the same metric through the public API
(``TorchBlockDataPlane.save_gather(..., digests=...)`` and ``load_scatter``,
one pinned allocation per block as the host tier uses), host wall time
including table uploads and the CRC / digest read-back. Both directions also
appear as fractions of a contiguous pinned cudaMemcpy timed in the same run.
Inputs (1.2 GB a step) exceed the 126 MB L2, so no flush is needed between steps.

With N GPUs (torchrun) every rank runs its own session on its own GPU: the
shards are independent (weak scaling), no collective touches the data path.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "KV save/restore GB/s per GPU vs host-link+HBM roofline; 8k Qwen3-8B restore ms"
UNIT = "GB/s"
LAYERS, HEADS, HEAD_DIM, BLOCK = 36, 8, 128, 16
PEAKS = ROOT / "MEASURED_PEAKS.json"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--pool-blocks", type=int, default=32768)
    p.add_argument("--layers", type=int, default=LAYERS)
    p.add_argument("--heads", type=int, default=HEADS, help="KV heads a rank holds")
    p.add_argument("--model", choices=["qwen3-8b", "qwen3-32b-tp"], default="qwen3-8b",
                   help="qwen3-32b-tp: benchmark configuration 5, each of N ranks saves and restores its 8/N-head shard "
                        "of a 32768-token Qwen3-32B session (64 layers)")
    p.add_argument("--ctas", type=int, default=0, help="CTAs for the data-plane kernels (0: library default)")
    p.add_argument("--restore-mode", choices=["direct", "staged"], default="staged")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-shard", action="store_true",
                   help="skip the sharded (BASELINE config 5) and regroup sub-objects of the session line")
    p.add_argument("--explore", type=str, default="", help="write a per-phase / CTA sweep breakdown to this path")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--workload", choices=["session", "disk", "reshard", "rotation", "kernels"], default="session",
                   help="session: benchmark configuration 2 (the default line); disk: configuration 3, verified restores of "
                        "8k and 32k-token snapshots from one pinned staging buffer with seeded corruption; "
                        "reshard: TP regroup over NVLink; rotation: configuration 4; kernels: the on-device "
                        "gather, scatter and CRC kernels alone against a torch device copy")
    p.add_argument("--blob-dir", type=str, default="",
                   help="where the disk workload writes its blob files (default: the system temp dir)")
    p.add_argument("--quick", action="store_true",
                   help="only the device-timed steps (a short run for profiling captures)")
    return p.parse_args()


def log(*args):
    print(*args, file=sys.stderr, flush=True)


# ---- clocks ----------------------------------------------------------------------------------

class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons while the timed region runs.

    The sampler starts early (its first sample can take a second or more with eight
    ranks starting it at once); ``begin`` and ``stop`` bound the timed region, and
    only samples that arrive inside it count.
    """
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        import threading
        self.proc, self.lines, self.t0 = None, [], None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line))

    def begin(self, wait=15.0):
        """Wait (bounded) for the sampler's first line, then open the timed window."""
        deadline = time.monotonic() + wait
        while self.proc is not None and not self.lines and time.monotonic() < deadline:
            time.sleep(0.05)
        self.t0 = time.monotonic()

    def stop(self):
        if self.proc is None:
            return {"unavailable": "nvidia-smi not found"}
        t1 = time.monotonic()
        time.sleep(0.25)                      # let a sample taken inside the window arrive
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.reader.join(timeout=5)
        t0 = self.t0 if self.t0 is not None else t1
        inside = [line for t, line in self.lines if t0 <= t <= t1 + 0.25]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in inside:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, value in zip(names, parts[2:]):
                if value.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"unavailable": "no samples"}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def smi_index(local):
    """nvidia-smi's index of this rank's GPU (CUDA_VISIBLE_DEVICES may renumber them)."""
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = [p.strip() for p in visible.split(",") if p.strip()]
    if local < len(parts) and parts[local].isdigit():
        return int(parts[local])
    return local


# ---- distributed plumbing ----------------------------------------------------------------------

def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- the workload --------------------------------------------------------------------------------

def make_caches(args, device):
    import torch
    gen = torch.Generator(device=device)
    caches = {}
    for i in range(args.layers):
        gen.manual_seed(args.seed * 1000 + i)
        t = torch.empty((2, args.pool_blocks, BLOCK, args.heads, HEAD_DIM), dtype=torch.bfloat16, device=device)
        t.normal_(generator=gen)
        caches[f"model.layers.{i}.self_attn.attn"] = t
    return caches


def session_blocks(args, n):
    """Two disjoint seeded block sets of n blocks each (save, restore); block 0 is kept free."""
    import numpy as np
    if args.pool_blocks < 2 * n + 1:
        raise SystemExit(f"--pool-blocks {args.pool_blocks} is too small: two disjoint {n}-block sessions "
                         f"need at least {2 * n + 1}")
    order = np.random.Generator(np.random.PCG64(args.seed + 17)).permutation(args.pool_blocks - 1) + 1
    return [int(b) for b in order[:n]], [int(b) for b in order[n:2 * n]]


def pinned_copy_peaks(nbytes, device, repeats=5):
    """A contiguous pinned <-> device cudaMemcpy of the session's size, timed with events (best of 5)."""
    import torch
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    stream = torch.cuda.Stream(device)
    out = {}
    for name, (dst, src) in {"h2d": (dev, host), "d2h": (host, dev)}.items():
        best = float("inf")
        for _ in range(repeats + 1):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                start.record()
                dst.copy_(src, non_blocking=True)
                end.record()
            end.synchronize()
            best = min(best, start.elapsed_time(end))
        out[name] = nbytes / (best / 1e3) / 1e9
    del dev, host
    return out


def duplex_box_peak(nbytes, device, world, repeats=3):
    """Every rank at once: pinned H2D and D2H cudaMemcpy of the session's size on two streams.

    Barrier-aligned and timed with events on each rank (max over ranks, best of
    ``repeats``); returns the box's aggregate GB/s, both directions summed. This is
    the ceiling the whole save + restore pipeline shares: on one GPU its full-duplex
    link, on several GPUs also the host memory and PCIe switches they share.
    """
    import torch
    dev_in = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dev_out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    host_in = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host_out = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    best = float("inf")
    for _ in range(repeats + 1):
        torch.cuda.synchronize()
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        start.record(up)
        down.wait_event(start)
        with torch.cuda.stream(up):
            dev_in.copy_(host_in, non_blocking=True)
        with torch.cuda.stream(down):
            host_out.copy_(dev_out, non_blocking=True)
        done = torch.cuda.Event()
        done.record(down)
        up.wait_event(done)
        end = torch.cuda.Event(enable_timing=True)
        end.record(up)
        end.synchronize()
        best = min(best, max_over_ranks(start.elapsed_time(end), world))
    del dev_in, dev_out, host_in, host_out
    return world * 2 * nbytes / (best / 1e3) / 1e9


class Engine:
    """The data plane's kernels launched straight through the C ABI with resident tables.

    A stream of sessions through one GPU, three deep. Step k saves session k and
    restores session k-1 (the snapshot step k-1 saved) into other blocks, the way
    the connector's save and load threads overlap on a serving worker:

    * copy stream: gather session k into device staging (CRC32C fused), then the
      copy engine moves it to pinned memory (device to host);
    * SHA stream k%2: SHA-256 of the staged blocks (the store's content ids);
    * load stream: the scatter kernel reads snapshot k-1 from pinned memory in
      place (host to device) and writes it into the restore blocks, checking
      every block's CRC32C against the one its save computed.

    The host link is full duplex, so the two copy directions overlap; staging,
    snapshots and CRCs rotate through three buffers and every reuse waits on an event.
    """

    def __init__(self, plane, save_ids, restore_ids, ctas, restore_mode):
        import torch
        from kvsnap_b200.dataplane import _dp
        self.torch = torch
        self.plane = plane
        self.lib = _dp(plane.pool.lib)
        self.spans = plane._spans()
        self.copy = plane._scatter_targets()
        self.load = plane._load_stream
        self.load_copy = plane._load_copy_stream
        self.sides = plane._sha_streams
        self.chunk = max(1, (64 << 20) // plane.block_bytes)
        self.n = len(save_ids)
        self.size = plane.block_bytes
        # As the API launches them: beside SHA-256 kernels, the device-memory kernels leave their SMs free.
        self.ctas = ctas or plane.hbm_ctas
        self.restore_mode = restore_mode
        dev = plane._device()
        n, size = self.n, self.size
        i64 = dict(dtype=torch.int64, device=dev)
        self.depth = 3
        self.stage = [torch.empty(n * size, dtype=torch.uint8, device=dev) for _ in range(self.depth)]
        self.snapshot = [plane.pool.reserve(n * size) for _ in range(self.depth)]
        self.stage_addrs = [torch.tensor([st.data_ptr() + i * size for i in range(n)], **i64) for st in self.stage]
        self.pinned_addrs = [torch.tensor([sn.pointer + i * size for i in range(n)], **i64) for sn in self.snapshot]
        if restore_mode == "staged":
            self.stage_in = torch.empty(n * size, dtype=torch.uint8, device=dev)
            self.stage_in_addrs = torch.tensor([self.stage_in.data_ptr() + i * size for i in range(n)], **i64)
        self.save_ids = torch.tensor(save_ids, **i64)
        self.restore_ids = torch.tensor(restore_ids, **i64)
        self.crc = [torch.empty(n, dtype=torch.int32, device=dev) for _ in range(self.depth)]
        self.crc_restore = torch.empty(n, dtype=torch.int32, device=dev)
        self.digest = [torch.empty(n * 32, dtype=torch.uint8, device=dev) for _ in range(self.depth)]
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.handle = plane.pool.handle
        self.k = 0
        self.events = {}
        self.launches_per_step = 0

    def _ok(self, rc):
        if rc < 0:
            raise RuntimeError(self.plane.pool.lib.kvsnap_cuda_error().decode())

    def _event(self, name, k, stream, timing=False):
        e = self.torch.cuda.Event(enable_timing=timing)
        e.record(stream)
        self.events[(name, k)] = e
        return e

    def _wait(self, stream, name, k):
        e = self.events.get((name, k))
        if e is not None:
            stream.wait_event(e)

    def step(self, marks=None):
        torch, lib, n, size = self.torch, self.lib, self.n, self.size
        k, b, depth = self.k, self.k % self.depth, self.depth
        nspans = len(self.plane.layers)
        timing = marks is not None
        launches = 0
        side = self.sides[k % len(self.sides)]
        # ---- save session k ----
        self._wait(self.copy, "hashed", k - depth)          # staging[b] free
        self._wait(self.copy, "restored", k - depth + 1)    # snapshot[b] and crc[b] read by restore(k-depth+1)
        t0 = self._event("t0", k, self.copy, timing)
        self._ok(lib.kvsnap_dp_gather(self.spans.data_ptr(), nspans, size, self.save_ids.data_ptr(),
                                      self.stage_addrs[b].data_ptr(), n, 0, self.crc[b].data_ptr(),
                                      self.status.data_ptr(), 16 | self.plane._hbm, self.ctas, self.copy.cuda_stream))
        launches += 2   # gather + CRC finish
        gathered = self._event("gathered", k, self.copy, timing)
        side.wait_event(gathered)
        s0 = self._event("sha0", k, side, timing)
        self._ok(lib.kvsnap_dp_sha256(self.stage_addrs[b].data_ptr(), n, size, self.digest[b].data_ptr(),
                                      side.cuda_stream))
        launches += 1
        self._event("hashed", k, side, timing)
        self._ok(lib.kvsnap_pool_copy(self.handle, self.snapshot[b].ident, 0, self.stage[b].data_ptr(), n * size, 1,
                                      self.copy.cuda_stream))
        self._event("saved", k, self.copy, timing)
        # ---- restore session k-1 (its snapshot and CRCs), concurrently ----
        r0 = None
        if ("saved", k - 1) in self.events:
            p = (k - 1) % depth
            self._wait(self.load, "saved", k - 1)
            self._wait(self.load_copy, "saved", k - 1)
            self._wait(self.load_copy, "restored", k - 1)   # stage_in free
            r0 = self._event("r0", k, self.load_copy, timing)
            if self.restore_mode == "staged":
                # Copy engine into device staging chunk by chunk, each chunk scattered
                # (and its CRCs checked) from HBM as soon as it lands.
                for first in range(0, n, self.chunk):
                    last = min(n, first + self.chunk)
                    self._ok(lib.kvsnap_pool_copy_on(self.handle, self.snapshot[p].ident, first * size,
                                                     self.stage_in.data_ptr() + first * size, (last - first) * size,
                                                     0, self.load_copy.cuda_stream))
                    landed = torch.cuda.Event()
                    landed.record(self.load_copy)
                    self.load.wait_event(landed)
                    self._ok(lib.kvsnap_dp_scatter(self.spans.data_ptr(), nspans, size,
                                                   self.stage_in_addrs[first:].data_ptr(),
                                                   self.restore_ids[first:].data_ptr(), last - first,
                                                   self.crc_restore[first:].data_ptr(), self.crc[p][first:].data_ptr(),
                                                   0, self.status.data_ptr(), 16 | self.plane._hbm, self.ctas,
                                                   self.load.cuda_stream))
                    launches += 2   # scatter + CRC verify finish
            else:
                self.load.wait_event(self.events[("r0", k)])
                self._ok(lib.kvsnap_dp_scatter(self.spans.data_ptr(), nspans, size, self.pinned_addrs[p].data_ptr(),
                                               self.restore_ids.data_ptr(), n, self.crc_restore.data_ptr(),
                                               self.crc[p].data_ptr(), 0, self.status.data_ptr(), 16,
                                               self.plane.host_ctas, self.load.cuda_stream))
                launches += 2   # scatter + CRC verify finish
            self._event("restored", k, self.load, timing)
        if timing:
            marks.append((k, r0 is not None))
        self.launches_per_step = launches
        self.k += 1

    def gather_only(self):
        """One save gather (KV -> device staging, tail zeroing, CRC32C) on the copy stream."""
        self._ok(self.lib.kvsnap_dp_gather(self.spans.data_ptr(), len(self.plane.layers), self.size,
                                           self.save_ids.data_ptr(), self.stage_addrs[0].data_ptr(), self.n, 0,
                                           self.crc[0].data_ptr(), self.status.data_ptr(), 16 | self.plane._hbm,
                                           self.ctas, self.copy.cuda_stream))

    def scatter_only(self):
        """One restore scatter (device staging -> KV, CRC32C checked) on the copy stream."""
        self._ok(self.lib.kvsnap_dp_scatter(self.spans.data_ptr(), len(self.plane.layers), self.size,
                                            self.stage_addrs[0].data_ptr(), self.restore_ids.data_ptr(), self.n,
                                            self.crc_restore.data_ptr(), self.crc[0].data_ptr(), 0,
                                            self.status.data_ptr(), 16 | self.plane._hbm, self.ctas,
                                            self.copy.cuda_stream))

    def join(self):
        """Make the copy stream wait for everything queued on the other streams."""
        for stream in (self.load, self.load_copy, *self.sides):
            e = self.torch.cuda.Event()
            e.record(stream)
            self.copy.wait_event(e)

    def phases(self, marks):
        """Mean device time of each phase over the timed steps."""
        out = {"gather": [], "sha256": [], "d2h": [], "restore": [], "save_latency": []}
        for k, restored in marks:
            ev = lambda name: self.events[(name, k)]   # noqa: E731
            out["gather"].append(ev("t0").elapsed_time(ev("gathered")))
            out["sha256"].append(ev("sha0").elapsed_time(ev("hashed")))
            out["d2h"].append(ev("gathered").elapsed_time(ev("saved")))
            out["save_latency"].append(max(ev("t0").elapsed_time(ev("saved")), ev("t0").elapsed_time(ev("hashed"))))
            if restored:
                out["restore"].append(ev("r0").elapsed_time(ev("restored")))
        return {key: statistics.mean(v) for key, v in out.items() if v}


def check_session(plane, save_ids, restore_ids, tokens):
    """Size-independent parity at full size: the restored blocks re-save to the same content ids and
    CRCs as the saved ones, and a sample of blocks hashes on the host (hashlib, native CRC) to them."""
    import hashlib
    from kvsnap_b200.crc32c import crc32c
    n, size = len(save_ids), plane.block_bytes
    with plane.staging(n) as a, plane.staging(n) as b:
        first, second = [], []
        plane.save_gather(save_ids, [(a, i * size) for i in range(n)], tokens, digests=first)
        plane.save_gather(restore_ids, [(b, i * size) for i in range(n)], tokens, digests=second)
        if first != second:
            raise AssertionError("restored blocks differ from the saved ones")
        for i in (0, n // 2, n - 1):
            block = a.read_range(i * size, size)
            if (hashlib.sha256(block).hexdigest(), crc32c(block)) != first[i]:
                raise AssertionError(f"GPU digest of block {i} differs from the host's")
    return True


def reference_gpu(caches, save_ids, restore_ids, tokens, reps=5):
    """The reference's own GPU data plane on this GPU, the same cache and session as ours.

    kvsnap's stock ``TorchBlockDataPlane`` (installed under baseline/_ref with
    its CUDA pool): the save gathers with torch ``index_select`` + ``cat`` a
    64 MiB chunk at a time and copies each chunk to pinned memory, then zeroes
    the last block's tail on the host (kvsnap/connector/dataplane.py:388-437);
    the restore is its Triton kernel reading pinned memory
    (kvsnap/connector/copy_kernel.py:23-49). Timed on the host around each call
    (both wait for their copies), one session at a time, one pinned buffer for
    the session (the disk tier's target). Returns a dict, or the reason it
    could not run.
    """
    import torch
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "kvsnap" / "_native").is_dir():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    if str(ref) not in sys.path:
        sys.path.append(str(ref))
    saved_env = os.environ.pop("KVSNAP_CUDA_LIBRARY", None)
    try:
        from kvsnap.connector import dataplane as theirs
        from kvsnap_b200.dataplane import _split_paged
        block_bytes = sum(2 * t[0, 0].numel() * t.element_size() for t in caches.values())   # K and V
        plane = theirs.TorchBlockDataPlane(_split_paged(caches, BLOCK), BLOCK,
                                           (len(save_ids) + 4) * block_bytes + (64 << 20))
    except Exception as exc:                                      # noqa: BLE001 - reported, not fatal
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    finally:
        if saved_env is not None:
            os.environ["KVSNAP_CUDA_LIBRARY"] = saved_env
    try:
        plane.warm_up()
        n, size = len(save_ids), plane.block_bytes
        with plane.staging(n) as snap:
            targets = [(snap, i * size) for i in range(n)]
            saves, restores = [], []
            for _ in range(reps + 1):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                plane.save_gather(save_ids, targets, tokens)
                saves.append((time.perf_counter() - t0) * 1e3)
                t0 = time.perf_counter()
                plane.load_scatter(restore_ids, targets)
                restores.append((time.perf_counter() - t0) * 1e3)
        save_ms, restore_ms = statistics.median(saves[1:]), statistics.median(restores[1:])
        return {"save_ms": round(save_ms, 3), "restore_ms": round(restore_ms, 3),
                "save_gbs": round(n * size / save_ms / 1e6, 2), "restore_gbs": round(n * size / restore_ms / 1e6, 2),
                "how": "kvsnap TorchBlockDataPlane from baseline/_ref: torch index_select+cat and cudaMemcpyAsync "
                       "save, Triton restore kernel; one session at a time, one pinned buffer"}
    except Exception as exc:                                      # noqa: BLE001
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
    finally:
        plane.close()


# ---- the reference's CPU path ----------------------------------------------------------------------

class ReferenceCPU:
    """The reference's own host path on a bounded sample of the workload, timed on this host's cores.

    With the reference installed under baseline/_ref (kind "reference"), its
    unmodified ``TorchBlockDataPlane`` runs on CPU tensors through the CUDA-free
    stand-ins of ``oracle/refharness.py``: ``save_gather`` gathers with torch
    ``index_select`` + ``cat`` and zeroes the last block's tail on the host
    (kvsnap/connector/dataplane.py:388-437), the store hashes the packed blocks
    with its own ``_prepare_payloads`` (SHA-256 and its compiled CRC32C on 8
    threads, kvsnap/store/store.py:616-629), and ``load_scatter`` moves each
    (block, layer) span the way its restore kernel does. Without it (kind
    "port"): the same steps restated with torch, the oracle's CRC32C and
    ``hashlib``. The cache is a ``pool_blocks`` Qwen3-8B pool in host memory,
    far beyond the CPU caches, built once; each pass saves ``sample_blocks``
    blocks (``ids``, seeded random ones by default) and restores them into
    ``back``.
    """

    def __init__(self, sample_blocks, threads, layers=LAYERS, pool_blocks=1100, ids=None, back=None, tokens=None):
        import numpy as np
        import torch
        torch.set_num_threads(threads)
        self.threads, self.sample_blocks, self.pool_blocks = threads, sample_blocks, pool_blocks
        caches = {}
        for i in range(layers):
            t = torch.empty((2, pool_blocks, BLOCK, HEADS, HEAD_DIM), dtype=torch.bfloat16)
            t.view(torch.int16).fill_(0x1234 + i)
            caches[f"model.layers.{i}.self_attn.attn"] = t
        if ids is None:
            order = np.random.Generator(np.random.PCG64(11)).permutation(pool_blocks - 1) + 1
            ids = [int(b) for b in order[:sample_blocks]]
            back = [int(b) for b in order[sample_blocks:2 * sample_blocks]]
        tokens = sample_blocks * BLOCK - 5 if tokens is None else tokens
        ref = ROOT / "baseline" / "_ref"
        if (ref / "kvsnap" / "_native").is_dir():
            self.kind = "reference"
            if str(ref) not in sys.path:
                sys.path.append(str(ref))
            from unittest.mock import patch
            from kvsnap.connector import dataplane as theirs
            from kvsnap.store import store as their_store
            from kvsnap_b200.dataplane import _split_paged
            from oracle.refharness import HostBuffer, register, restore_by_memmove
            plane = register(theirs, _split_paged(caches, BLOCK), BLOCK)
            self.size = size = plane.block_bytes
            targets = [(HostBuffer(size), 0) for _ in ids]      # reused, as the connector reuses pinned memory

            def one_pass():
                plane.save_gather(ids, targets, tokens)
                their_store._prepare_payloads([a.read_range(0, size) for a, _ in targets])
                with patch.object(theirs, "copy_host_blocks", new=restore_by_memmove):
                    plane.load_scatter(back, targets)
        else:
            import ctypes
            import hashlib
            self.kind = "port"
            from oracle import oracle as port
            crc_fn = port._lib().oracle_crc32c
            crc_fn.argtypes, crc_fn.restype = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32], ctypes.c_uint32
            rows = [t[k].view(pool_blocks, -1).view(torch.int64) for t in caches.values() for k in range(2)]
            span_words = rows[0].shape[1]
            self.size = len(rows) * span_words * 8
            id_t, back_t = torch.tensor(ids), torch.tensor(back)

            def digest(block):
                view = block.numpy()
                return hashlib.sha256(view).hexdigest(), crc_fn(view.ctypes.data, view.nbytes, 0)

            def one_pass():
                stage = torch.cat([r.index_select(0, id_t) for r in rows], dim=1)
                with ThreadPoolExecutor(max_workers=8) as hashers:
                    list(hashers.map(digest, list(stage)))
                offset = 0
                for r in rows:
                    r.index_copy_(0, back_t, stage[:, offset:offset + span_words])
                    offset += span_words
        self.one_pass = one_pass
        one_pass()                                      # the pool's pages and the thread pools warm

    def run(self, seconds):
        """Passes for at least ``seconds`` (at least one); GB/s of saved + restored bytes."""
        done, start = 0, time.perf_counter()
        while True:
            self.one_pass()
            done += 1
            if time.perf_counter() - start >= seconds:
                break
        elapsed = time.perf_counter() - start
        moved = done * 2 * self.sample_blocks * self.size
        return {"value": moved / elapsed / 1e9, "unit": UNIT, "cores": self.threads, "kind": self.kind,
                "sample": f"{done} passes of save ({self.sample_blocks} Qwen3-8B blocks of {self.size} B from a "
                          f"{self.pool_blocks}-block host pool: the reference's save_gather, its store's SHA-256 + "
                          f"CRC32C on 8 threads) + restore (its load_scatter), {elapsed:.1f} s, {self.threads} "
                          f"torch threads"}


def run_reference(args, world, rank):
    """``--impl reference``: the reference's own CPU path on this workload, rank 0 only.

    Each step saves the session our arm saves (the same seeded block ids in a
    pool of ``--pool-blocks`` blocks, in host memory) through the reference's
    ``save_gather`` and store hashing, and restores it through its
    ``load_scatter`` (see ``ReferenceCPU``), on every host thread.
    """
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    n = (args.tokens + BLOCK - 1) // BLOCK
    # The pool lives in host memory here: on a host with too little free memory for the configured pool,
    # the largest one that fits in 60 % of it (the config line then records that size).
    block = args.layers * 2 * BLOCK * args.heads * HEAD_DIM * 2
    free = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    fits = int(0.6 * free) // block
    if fits < args.pool_blocks:
        if fits < 2 * n + 1:
            raise SystemExit(f"host memory holds {fits} blocks; the session needs a pool of {2 * n + 1}")
        log(f"host memory: pool of {fits} blocks instead of {args.pool_blocks}")
        args.pool_blocks = fits
    save_ids, restore_ids = session_blocks(args, n)
    t_setup = time.perf_counter()
    cpu = ReferenceCPU(n, threads, layers=args.layers, pool_blocks=args.pool_blocks, ids=save_ids,
                       back=restore_ids, tokens=args.tokens)
    log(f"reference CPU setup {time.perf_counter() - t_setup:.1f} s ({cpu.kind})")
    for _ in range(args.warmup):
        cpu.run(0.0)
    values, t0 = [], time.perf_counter()
    for _ in range(args.steps):
        values.append(cpu.run(0.0))
    elapsed = time.perf_counter() - t0
    value = cpu.sample_blocks * cpu.size * 2 * args.steps / elapsed / 1e9
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic", "impl": "reference",
            "config": session_config(args, n, cpu.size),
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": cpu.kind,
                             "sample": f"every step the whole session: {values[-1]['sample']}"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def session_config(args, n, size):
    """The ``config`` of the session workload (BASELINE config 2 by default)."""
    return {"workload": ("qwen3-8b 8k-token session save+restore (BASELINE config 2)" if args.model == "qwen3-8b"
                         else f"qwen3-32b 32k-token session, TP shard a rank (BASELINE config 5)"),
            "layers": args.layers, "kv_heads": args.heads, "head_dim": HEAD_DIM, "block_size": BLOCK,
            "pool_blocks": args.pool_blocks, "session_blocks": n, "session_bytes": n * size,
            "l2": "inputs (1.2 GB a step) larger than L2; no flush", "kv": "bf16, seeded"}


# ---- main ----------------------------------------------------------------------------------------------

def main():
    args = parse()
    world, rank, local = dist_setup() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    import torch
    from kvsnap_b200.dataplane import TorchBlockDataPlane

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.model == "qwen3-32b-tp":
        if 8 % world:
            raise SystemExit("qwen3-32b-tp needs 1, 2, 4 or 8 ranks")
        args.layers, args.heads, args.tokens = 64, 8 // world, 32768
        args.pool_blocks = max(args.pool_blocks if args.pool_blocks != 32768 else 0, 2 * 2048 + 64)
    if args.workload == "disk":
        run_disk(args, world, rank, device)
        return
    if args.workload == "reshard":
        run_reshard(args, world, rank, device)
        return
    if args.workload == "rotation":
        run_rotation(args, world, rank, device)
        return
    if args.workload == "kernels":
        run_kernels(args, world, rank, device)
        return
    n = (args.tokens + BLOCK - 1) // BLOCK
    t_setup = time.perf_counter()
    caches = make_caches(args, device)
    save_ids, restore_ids = session_blocks(args, n)
    size_guess = args.layers * 2 * BLOCK * args.heads * HEAD_DIM * 2
    plane = TorchBlockDataPlane(caches, BLOCK, 7 * n * size_guess + (64 << 20), restore_mode=args.restore_mode,
                                ctas=args.ctas)
    plane.warm_up()
    size = plane.block_bytes
    session = n * size
    torch.cuda.synchronize()
    log(f"setup {time.perf_counter() - t_setup:.1f} s; block {size} B, session {session} B")

    link = pinned_copy_peaks(session, device)
    box_duplex = duplex_box_peak(session, device, world)
    engine = Engine(plane, save_ids, restore_ids, args.ctas, args.restore_mode)

    # Device-timed steps: a stream of sessions, each step saving one and restoring the previous.
    clocks = Clocks(smi_index(local))
    for _ in range(max(1, args.warmup)):
        engine.step()
    torch.cuda.synchronize()
    if int(engine.status.item()) != 0:
        raise RuntimeError(f"kernel status {int(engine.status.item())} (CRC mismatch or bad table)")
    barrier(world)
    marks = []
    torch.cuda.synchronize()
    clocks.begin()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(engine.copy)
    for stream in (engine.load, engine.load_copy, *engine.sides):
        stream.wait_event(start)
    for _ in range(args.steps):
        engine.step(marks)
    engine.join()
    end.record(engine.copy)
    torch.cuda.synchronize()
    barrier(world)
    clock_info = clocks.stop()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    phases = engine.phases(marks)
    if int(engine.status.item()) != 0:
        raise RuntimeError(f"kernel status {int(engine.status.item())} during the timed steps")
    if args.quick:
        if rank == 0:
            print(json.dumps({"quick": True, "ms_per_step": round(ms, 3),
                              "phases_ms": {k: round(v, 3) for k, v in phases.items()}}), flush=True)
        for snap in engine.snapshot:
            snap.close()
        plane.close()
        return

    # The on-device kernels alone, back to back, for their rooflines (HBM read + write per launch).
    kernel_ms = {}
    for name, fn in (("gather", engine.gather_only), ("scatter", engine.scatter_only)):
        fn()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(engine.copy)
        for _ in range(10):
            fn()
        s1.record(engine.copy)
        torch.cuda.synchronize()
        kernel_ms[name] = max_over_ranks(s0.elapsed_time(s1) / 10, world)
    del fn                                               # a bound method of the engine: it holds the cache

    # End to end through the public API, host tier (one pinned allocation per block), with the
    # connector's threads: two save workers (vllm.py:202) and one load worker (vllm.py:203). Session k
    # is saved into snapshot k % 3 the way the drop-in connector saves: save_gather returns once the
    # blocks are in pinned memory (PendingDigests), and the save worker then collects the content ids
    # and CRCs the store needs. Session k is restored once save_gather has returned for it; a
    # snapshot is reused once its digests are in and its restore is done.
    from kvsnap_b200.dataplane import PendingDigests
    sets = [[plane.pool.reserve(size) for _ in range(n)] for _ in range(3)]
    places = [[(a, 0) for a in owned] for owned in sets]
    savers, loader = ThreadPoolExecutor(max_workers=2), ThreadPoolExecutor(max_workers=1)

    def save_session(k, landed):
        pending = PendingDigests()
        try:
            plane.save_gather(save_ids, places[k % 3], args.tokens, digests=pending)
        finally:
            landed.set()                             # a failed save surfaces through its future
        return pending.result()

    def run_sessions(first, count):
        saves, landed, restores = {}, {}, []
        for k in range(first, first + count):
            if k - 3 in saves:                       # snapshot k % 3 is free once its restore is done
                saves.pop(k - 3).result()
                while restores and restores[0][0] <= k - 3:
                    restores.pop(0)[1].result()
            landed[k] = threading.Event()
            saves[k] = savers.submit(save_session, k, landed[k])
            if k - 1 >= first:
                landed[k - 1].wait()
                restores.append((k - 1, loader.submit(plane.load_scatter, restore_ids, places[(k - 1) % 3])))
        last = first + count - 1
        landed[last].wait()
        restores.append((last, loader.submit(plane.load_scatter, restore_ids, places[last % 3])))
        for _, f in restores:
            f.result()
        for f in saves.values():
            f.result()

    run_sessions(0, max(2, args.warmup))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    run_sessions(0, args.steps)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) / args.steps * 1e3, world)
    savers.shutdown()
    loader.shutdown()
    for owned in sets:
        for a in owned:
            a.close()
    digests_ok = check_session(plane, save_ids, restore_ids, args.tokens)

    # One session at a time through the API: restore latency; save latency until the
    # blocks are in pinned memory (when save_gather returns) and until their digests are.
    from kvsnap_b200.dataplane import PendingDigests
    with plane.staging(n) as snap:
        places = [(snap, i * size) for i in range(n)]
        save_times, digest_times, restore_times = [], [], []
        for _ in range(max(3, args.steps // 2)):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            pending = PendingDigests()
            plane.save_gather(save_ids, places, args.tokens, digests=pending)
            save_times.append((time.perf_counter() - t0) * 1e3)
            pending.result()
            digest_times.append((time.perf_counter() - t0) * 1e3)
            t0 = time.perf_counter()
            plane.load_scatter(restore_ids, places)
            restore_times.append((time.perf_counter() - t0) * 1e3)
    # The reference's own GPU path on the same GPU, cache and session, one session at a time.
    ref_gpu = reference_gpu(caches, save_ids, restore_ids, args.tokens)
    restore_ms = max_over_ranks(statistics.median(restore_times), world)
    save_ms = max_over_ranks(statistics.median(save_times), world)
    save_digests_ms = max_over_ranks(statistics.median(digest_times), world)

    explore = {}
    if args.explore and rank == 0:
        explore = explore_phases(plane, engine, save_ids, restore_ids, link)
        Path(args.explore).write_text(json.dumps(explore, indent=1))


    peaks = json.loads(PEAKS.read_text()) if PEAKS.is_file() else {}
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if peaks else "fallback"
    value = world * 2 * session / (ms / 1e3) / 1e9
    e2e = world * 2 * session / (e2e_ms / 1e3) / 1e9
    restore_gbs = session / (phases["restore"] / 1e3) / 1e9
    gather_gbs = 2 * session / (kernel_ms["gather"] / 1e3) / 1e9
    scatter_gbs = 2 * session / (kernel_ms["scatter"] / 1e3) / 1e9
    d2h_gbs = session / (phases["d2h"] / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": dict(session_config(args, n, size), restore_mode=args.restore_mode),
        "phases_ms": {k: round(v, 3) for k, v in phases.items()},
        "restore_ms": round(restore_ms, 3),
        "save_ms": round(save_ms, 3),
        "save_digests_ms": round(save_digests_ms, 3),
        "host_link": {"h2d_memcpy_gbs": round(link["h2d"], 2), "d2h_memcpy_gbs": round(link["d2h"], 2),
                      "restore_gbs": round(restore_gbs, 2), "restore_frac": round(restore_gbs / link["h2d"], 3),
                      "save_d2h_gbs": round(d2h_gbs, 2), "save_frac": round(d2h_gbs / link["d2h"], 3),
                      "note": "per-phase rates measured while the other direction runs concurrently",
                      "restore_alone_frac": round(session / (restore_ms / 1e3) / 1e9 / link["h2d"], 3),
                      "save_alone_frac": round(session / (save_ms / 1e3) / 1e9 / link["d2h"], 3),
                      "alone_note": "one session at a time through the API (restore_ms, save_ms) over the "
                                    "pinned cudaMemcpy of the same bytes",
                      "box_duplex_gbs": round(box_duplex, 2), "value_frac_of_box_duplex": round(value / box_duplex, 3),
                      "box_note": "every rank's pinned H2D and D2H cudaMemcpy at once, both directions summed: "
                                  "the ceiling the whole-job value shares"},
        "roofline": {"bound": "hbm", "kernel": "span_kernel_hbm<gather>: KV -> device staging, tail zero, CRC32C",
                     "achieved": round(gather_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(gather_gbs / hbm_peak, 3),
                     **captured_traffic("span_kernel_hbm<gather> qwen3-8b 512 blocks", args, n),
                     "algorithmic_bytes": 2 * session, "ms": round(kernel_ms["gather"], 4),
                     "launch": f"{engine.ctas} CTAs", "peak_source": f"{peak_src} hbm_gbs (burst copy)"},
        "roofline_scatter": {"bound": "hbm", "kernel": "span_kernel_hbm<scatter>: device staging -> KV, CRC32C check",
                             "achieved": round(scatter_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                             "frac": round(scatter_gbs / hbm_peak, 3),
                             **captured_traffic("span_kernel_hbm<scatter> qwen3-8b 512 blocks", args, n),
                             "ms": round(kernel_ms["scatter"], 4)},
        "sha256_gbs": round(session / (phases["sha256"] / 1e3) / 1e9, 2),
        "e2e": {"value": round(e2e, 3), "unit": UNIT, "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": session + 16 * n, "d2h_bytes_per_step": session + 36 * n},
        "gpu_launches": engine.launches_per_step * args.steps,
        "clocks": clock_info,
        "parity": {"restored_equals_saved": digests_ok, "host_hash_sample": True},
        "reference_gpu": dict(ref_gpu, ours_save_ms=round(save_ms, 3), ours_restore_ms=round(restore_ms, 3),
                              note="both until the packed blocks are in pinned memory (save) or in the cache "
                                   "(restore); ours also computes CRC32C on the way and SHA-256 after"),
    }
    for snap in engine.snapshot:
        snap.close()
    plane.close()
    del engine, plane, caches
    release_device_memory()
    if not args.no_shard:
        # Benchmark configuration 5 on the same ranks: every rank's own TP-N shard, then (an even N) the
        # regroup of a TP-N snapshot restored at TP-N/2 over NVLink.
        line["sharded"] = measure_sharded(args, world, rank, device, box_duplex)
        if world >= 2 and world % 2 == 0:
            line["reshard"] = measure_reshard(args, world, rank, device)
    if rank == 0 and world == 1 and not args.no_cpu:
        # Last, so that its host-memory traffic touches no GPU measurement: the whole session from the
        # CPU arm's own host pool (its seeded block ids), for 10 s.
        line["cpu_baseline"] = ReferenceCPU(n, os.cpu_count() or 1, pool_blocks=max(1100, 2 * n + 1),
                                            tokens=args.tokens).run(10.0)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def captured_traffic(kernel, args, n):
    """``traffic`` of a roofline field: DRAM read + write bytes per launch of ``kernel`` from its ncu capture
    (profiles/roofline_traffic.json, written from the summaries there), for the workload it was captured on."""
    path = ROOT / "profiles" / "roofline_traffic.json"
    entry = json.loads(path.read_text()).get(kernel) if path.is_file() else None
    if entry is None or args.model != "qwen3-8b" or args.layers != LAYERS or n != 512:
        return {"traffic": None, "traffic_note": "no ncu capture of this kernel on this workload"}
    return {"traffic": entry["dram_read_bytes"] + entry["dram_write_bytes"],
            "traffic_note": f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch ({entry['launch']}), "
                            f"{entry['summary']}"}


def release_device_memory():
    """Hand a finished workload's device memory back: its plane, pool and allocations refer to one another,
    so they go at a collection, and then the caching allocator returns the blocks to the device."""
    import gc
    import torch
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    free, total = torch.cuda.mem_get_info()
    log(f"device memory free {free / 2**30:.1f} of {total / 2**30:.1f} GiB")


def measure_sharded(args, world, rank, device, box_duplex):
    """Benchmark configuration 5: each rank's TP-N shard of a 32768-token Qwen3-32B session, all ranks at once.

    A rank holds 64 layers of 8/N KV heads (TP-N, kvsnap/connector/vllm.py:9-14)
    in a pool of 4160 blocks and saves and restores its 2048-block shard
    through the API, one pinned buffer a session, with content ids and CRCs
    from the GPU: no collective touches the data path. Times are the median of
    a few sessions, max over ranks; box figures are all ranks' bytes over that.
    """
    import numpy as np
    import torch
    from kvsnap_b200.dataplane import PendingDigests, TorchBlockDataPlane
    layers, heads, n, pool = 64, 8 // world, 2048, 2 * 2048 + 64
    gen = torch.Generator(device=device)
    caches = {}
    for i in range(layers):
        gen.manual_seed(args.seed * 1000 + 700 + i + 100 * rank)
        t = torch.empty((2, pool, BLOCK, heads, HEAD_DIM), dtype=torch.bfloat16, device=device)
        t.normal_(generator=gen)
        caches[f"model.layers.{i}.self_attn.attn"] = t
    size = layers * 2 * BLOCK * heads * HEAD_DIM * 2
    plane = TorchBlockDataPlane(caches, BLOCK, n * size + (64 << 20), ctas=args.ctas)
    plane.warm_up()
    order = np.random.Generator(np.random.PCG64(args.seed + 29)).permutation(pool - 1) + 1
    save_ids, restore_ids = [int(b) for b in order[:n]], [int(b) for b in order[n:2 * n]]
    saves, digests, restores = [], [], []
    with plane.staging(n) as snapshot:
        targets = [(snapshot, i * size) for i in range(n)]
        for rep in range(4):
            torch.cuda.synchronize()
            barrier(world)
            t0 = time.perf_counter()
            pending = PendingDigests()
            plane.save_gather(save_ids, targets, n * BLOCK, digests=pending)
            t1 = time.perf_counter()
            pending.result()
            t2 = time.perf_counter()
            barrier(world)
            t3 = time.perf_counter()
            plane.load_scatter(restore_ids, targets)
            t4 = time.perf_counter()
            if rep:                                          # the first is a warm-up
                saves.append(t1 - t0)
                digests.append(t2 - t0)
                restores.append(t4 - t3)
    plane.close()
    del plane, caches
    release_device_memory()
    save_s = max_over_ranks(statistics.median(saves), world)
    digest_s = max_over_ranks(statistics.median(digests), world)
    restore_s = max_over_ranks(statistics.median(restores), world)
    shard = n * size
    return {"config": f"qwen3-32b 32768-token session, TP-{world} shard a rank (BASELINE config 5)",
            "layers": layers, "kv_heads_per_rank": heads, "blocks": n, "shard_bytes_per_rank": shard,
            "save_ms": round(save_s * 1e3, 3), "save_digests_ms": round(digest_s * 1e3, 3),
            "restore_ms": round(restore_s * 1e3, 3),
            "save_gbs_per_gpu": round(shard / save_s / 1e9, 2), "restore_gbs_per_gpu": round(shard / restore_s / 1e9, 2),
            "save_gbs_box": round(world * shard / save_s / 1e9, 2),
            "restore_gbs_box": round(world * shard / restore_s / 1e9, 2),
            "box_duplex_gbs": round(box_duplex, 2),
            "note": "one session at a time a rank, all ranks at once; the box's ranks share its host link"}


def run_kernels(args, world, rank, device):
    """The on-device kernels alone on one session (HBM on both sides), each timed with CUDA events.

    Gather and scatter with and without CRC32C, the CRC of device blocks, and a torch
    device-to-device copy of the same bytes as the control: the fraction of the measured
    HBM copy rate each reaches (2 x bytes for the copies, 1 x bytes for the CRC alone).
    """
    import torch
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    n = (args.tokens + BLOCK - 1) // BLOCK
    caches = make_caches(args, device)
    save_ids, restore_ids = session_blocks(args, n)
    plane = TorchBlockDataPlane(caches, BLOCK, 64 << 20, ctas=args.ctas)
    plane.warm_up()
    lib, spans, nspans, size = plane.pool.lib, plane._spans(), len(plane.layers), plane.block_bytes
    total = n * size
    stage = torch.empty(total, dtype=torch.uint8, device=device)
    other = torch.empty_like(stage)
    addrs = torch.arange(n, dtype=torch.int64, device=device) * size + stage.data_ptr()
    ids = torch.tensor(save_ids, dtype=torch.int64, device=device)
    ids2 = torch.tensor(restore_ids, dtype=torch.int64, device=device)
    crc = torch.zeros(n, dtype=torch.int32, device=device)
    crc2 = torch.zeros(n, dtype=torch.int32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    hbm = 16 | plane._hbm

    def ok(rc):
        if rc != 0:
            raise RuntimeError(lib.kvsnap_cuda_error().decode())

    def gather(with_crc):
        ok(lib.kvsnap_dp_gather(spans.data_ptr(), nspans, size, ids.data_ptr(), addrs.data_ptr(), n, 0,
                                crc.data_ptr() if with_crc else 0, status.data_ptr(), hbm, args.ctas, stream))

    def scatter(with_crc):
        ok(lib.kvsnap_dp_scatter(spans.data_ptr(), nspans, size, addrs.data_ptr(), ids2.data_ptr(), n,
                                 crc2.data_ptr() if with_crc else 0, crc.data_ptr() if with_crc else 0, 0,
                                 status.data_ptr(), hbm, args.ctas, stream))

    def crc_only():
        ok(lib.kvsnap_dp_crc32c(addrs.data_ptr(), n, size, crc2.data_ptr(), crc.data_ptr(), status.data_ptr(),
                                hbm, args.ctas, stream))

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    peak = json.loads(PEAKS.read_text()).get("hbm_gbs", 6650.0) if PEAKS.is_file() else 6650.0
    gather(True)                  # the CRCs every later check compares against
    torch.cuda.synchronize()
    rows = {"torch_copy": (timed(lambda: other.copy_(stage)), 2),
            "gather_crc": (timed(lambda: gather(True)), 2),
            "gather_copy": (timed(lambda: gather(False)), 2),
            "scatter_crc": (timed(lambda: scatter(True)), 2),
            "scatter_copy": (timed(lambda: scatter(False)), 2),
            "crc_only": (timed(crc_only), 1)}
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError(f"kernel status {int(status.item())}: a verified scatter or CRC disagreed")
    if rank == 0:
        print(json.dumps({"workload": f"on-device kernels, {args.layers} layers x {args.heads} KV heads, "
                                      f"{n}-block session ({total} B)",
                          "steps": args.steps, "peak_gbs": peak,
                          "kernels": {k: {"ms": round(ms, 4), "gbs": round(m * total / ms / 1e6, 1),
                                          "frac": round(m * total / ms / 1e6 / peak, 3)}
                                      for k, (ms, m) in rows.items()}}), flush=True)
    plane.close()


def run_disk(args, world, rank, device):
    """Benchmark configuration 3: the disk tier's restore from one pinned staging buffer, CRC32C checked on the GPU.

    For 8192- and 32768-token Qwen3-8B snapshots: save the session into one
    staging buffer (its CRCs recorded, as the store's manifest does), flip one
    byte in a seeded 1-in-1000 of the blocks (at least one), and require the
    verified restore to name exactly those blocks and leave the cache untouched.
    Then time the verified restore of the repaired snapshot into fragmented
    (seeded random) block tables.
    """
    import ctypes
    import numpy as np
    import torch
    from kvsnap_b200.dataplane import CorruptBlockError, TorchBlockDataPlane
    caches = make_caches(args, device)
    rows = []
    size_guess = args.layers * 2 * BLOCK * HEADS * HEAD_DIM * 2
    # Two 32k-token snapshots' worth of pinned memory: the snapshot and the blob phase's staging.
    plane = TorchBlockDataPlane(caches, BLOCK, 2 * 2048 * size_guess + (256 << 20), ctas=args.ctas)
    plane.warm_up()
    size = plane.block_bytes
    rng = np.random.Generator(np.random.PCG64(args.seed + 33))
    for tokens in (8192, 32768):
        n = tokens // BLOCK
        order = rng.permutation(args.pool_blocks - 1) + 1
        saved, restored = [int(b) for b in order[:n]], [int(b) for b in order[n:2 * n]]
        with plane.staging(n) as staged:
            sources = [(staged, i * size) for i in range(n)]
            digests = []
            plane.save_gather(saved, sources, tokens, digests=digests)
            crcs = [c for _, c in digests]
            corrupt = sorted(set(int(i) for i in rng.choice(n, max(1, n // 1000), replace=False)))
            flips = []
            for i in corrupt:
                at = staged.pointer + i * size + int(rng.integers(size))
                flips.append(at)
                ctypes.memset(at, ctypes.string_at(at, 1)[0] ^ 0x5A, 1)
            before = []
            check_ids = restored[:8]
            with plane.staging(len(check_ids)) as probe:
                plane.save_gather(check_ids, [(probe, i * size) for i in range(len(check_ids))],
                                  len(check_ids) * BLOCK, digests=before)
            detected = None
            try:
                plane.load_scatter(restored, sources, expected_crc32c=crcs)
            except CorruptBlockError as exc:
                detected = exc.blocks
            after = []
            with plane.staging(len(check_ids)) as probe:
                plane.save_gather(check_ids, [(probe, i * size) for i in range(len(check_ids))],
                                  len(check_ids) * BLOCK, digests=after)
            for at in flips:
                ctypes.memset(at, ctypes.string_at(at, 1)[0] ^ 0x5A, 1)
            plane.load_scatter(restored, sources, expected_crc32c=crcs)       # warm
            torch.cuda.synchronize()
            times = []
            for _ in range(max(3, args.steps // 2)):
                t0 = time.perf_counter()
                plane.load_scatter(restored, sources, expected_crc32c=crcs)
                times.append((time.perf_counter() - t0) * 1e3)
            ms = statistics.median(times)
            row = {"tokens": tokens, "blocks": n, "bytes": n * size, "corrupted": corrupt,
                   "detected": detected, "detected_exactly": detected == corrupt,
                   "cache_untouched_on_failure": before == after,
                   "verified_restore_ms": round(ms, 3), "gbs": round(n * size / (ms / 1e3) / 1e9, 2)}
            row.update(blob_phase(plane, sources, digests, restored, n, size, args))
            restored_digests = []      # re-save the restored blocks over the snapshot and compare ids
            plane.save_gather(restored, sources, tokens, digests=restored_digests)
            row["restore_bit_exact"] = restored_digests == digests
            rows.append(row)
    if rank == 0:
        print(json.dumps({"workload": "disk-tier verified restore (BASELINE config 3)", "rows": rows}), flush=True)
    plane.close()


def blob_phase(plane, sources, digests, restored, n, size, args):
    """The same snapshot as KVSBLOB1 files: write_blobs, then restores from the files.

    Timed, with the files in the page cache (nothing here drops caches):
    * blob_write: write_blobs from the pinned snapshot ("process" durability: no fdatasync);
    * read_restore: read_and_restore, reads overlapped with GPU copies and CRC checks;
    * read_then_restore: the reference's order of work on the same files: every block read and
      CRC-checked on the host (8 threads, reference store.py:676-713), then load_scatter.
    Skipped (with the reason) when the file system lacks room for three copies of the snapshot.
    """
    import shutil
    import tempfile
    from concurrent.futures import ThreadPoolExecutor
    from kvsnap_b200 import blobs
    from kvsnap_b200.native_io import NativeIO, resolve_io_library
    root = args.blob_dir or tempfile.gettempdir()
    if shutil.disk_usage(root).free < 3 * n * size:
        return {"blobs": f"skipped: {root} has less than {3 * n * size} bytes free"}
    blob_dir = tempfile.mkdtemp(prefix="kvsnap-blobs-", dir=root)
    out = {}
    try:
        t0 = time.perf_counter()
        segments = blobs.write_blobs(blob_dir, sources, digests, size, durability="process")
        write_ms = (time.perf_counter() - t0) * 1e3
        io = NativeIO(resolve_io_library(), workers=8, queue_bytes=256 << 20)
        pipelined, serial = [], []
        with plane.staging(n) as staged:
            blobs.read_and_restore(plane, blob_dir, segments, restored, staged, io=io)      # warm
            for _ in range(3):
                t0 = time.perf_counter()
                blobs.read_and_restore(plane, blob_dir, segments, restored, staged, io=io)
                pipelined.append((time.perf_counter() - t0) * 1e3)

            def read_checked(i):
                address = staged.pointer + i * size
                blobs._read_block(io, blob_dir, segments[i], address, size)
                if io.crc32c_at(address, size) != segments[i]["crc32c"]:
                    raise RuntimeError("host CRC mismatch")

            targets = [(staged, i * size) for i in range(n)]
            with ThreadPoolExecutor(max_workers=8) as pool:
                for _ in range(3):
                    t0 = time.perf_counter()
                    list(pool.map(read_checked, range(n)))
                    plane.load_scatter(restored, targets)
                    serial.append((time.perf_counter() - t0) * 1e3)
        io.close()
        p_ms, s_ms = statistics.median(pipelined), statistics.median(serial)
        out = {"blob_files": len({s["blob_id"] for s in segments}),
               "blob_write_ms": round(write_ms, 2), "blob_write_gbs": round(n * size / (write_ms / 1e3) / 1e9, 2),
               "read_restore_ms": round(p_ms, 2), "read_restore_gbs": round(n * size / (p_ms / 1e3) / 1e9, 2),
               "read_then_restore_ms": round(s_ms, 2),
               "read_then_restore_gbs": round(n * size / (s_ms / 1e3) / 1e9, 2),
               "blob_note": "page-cache reads; read_then_restore is the reference's order: host CRC, then H2D"}
    finally:
        shutil.rmtree(blob_dir, ignore_errors=True)
    return out


def measure_reshard(args, world, rank, device):
    """Benchmark configuration 5's regroup: a TP-(2T) Qwen3-32B snapshot restored at TP-T over NVLink.

    World size W (torchrun, one GPU a rank): the snapshot was saved at TP=W (one
    shard a rank, 64 layers × 8/W heads, 2048 blocks = 32768 tokens), the cache
    it is restored into runs at TP=W/2 on ranks 0..W/2-1. Every rank copies its
    own shard from pinned memory into device memory it shares over CUDA IPC;
    each destination rank's regroup kernel reads its two shards (one its own,
    one a peer's over NVLink) and interleaves them into its cache blocks.
    Checked: sample blocks of every destination rank re-save to the interleave
    of the two shards' bytes (gathered from their ranks with NCCL).
    """
    import numpy as np
    import torch
    import torch.distributed as dist
    from kvsnap_b200.dataplane import TorchBlockDataPlane
    from kvsnap_b200.reshard import RegroupPlan, Regrouper
    if world < 2 or world % 2:
        raise SystemExit("the regroup workload needs an even number of ranks (torchrun --nproc-per-node 2|4|8)")
    plan = RegroupPlan(world, world // 2)
    layers, heads, n, pool = 64, 8, 2048, 4096
    dst_heads = heads // plan.dst_tp
    caches = {f"model.layers.{i}": torch.zeros((2, pool, BLOCK, dst_heads, HEAD_DIM), dtype=torch.bfloat16,
                                               device=device) for i in range(layers)}
    size = layers * 2 * BLOCK * dst_heads * HEAD_DIM * 2
    shard = size // plan.groups
    plane = TorchBlockDataPlane(caches, BLOCK, n * shard + size * 8 + (256 << 20), ctas=args.ctas)
    plane.warm_up()
    gen = torch.Generator(device=device).manual_seed(args.seed * 97 + rank)
    noise = torch.randint(0, 256, (n * shard,), dtype=torch.uint8, device=device, generator=gen)
    snapshot = plane.pool.reserve(n * shard)
    snapshot.copy(noise.data_ptr(), n * shard, 0, to_host=True)
    snapshot.wait()
    sources = [(snapshot, i * shard) for i in range(n)]
    order = np.random.Generator(np.random.PCG64(args.seed + 5)).permutation(pool - 1) + 1
    restored = [int(b) for b in order[:n]]
    regrouper = Regrouper(plane, plan, rank)
    regrouper.restore(restored, sources)                 # warm: shard buffer, IPC maps, kernels
    runs = []
    for _ in range(max(3, args.steps // 2)):
        torch.cuda.synchronize()
        dist.barrier()
        timings = {}
        t0 = time.perf_counter()
        regrouper.restore(restored, sources, timings=timings)
        timings["total_s"] = time.perf_counter() - t0
        runs.append(timings)
    regrouper.close()
    # Parity on sample blocks: destination rank r's packed block i = interleave of shards 2r, 2r+1.
    samples = [0, n // 2, n - 1]
    mine = torch.stack([noise[i * shard:(i + 1) * shard] for i in samples])
    gathered = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    ok = True
    if rank < plan.dst_tp:
        with plane.staging(len(samples)) as probe:
            plane.save_gather([restored[i] for i in samples], [(probe, j * size) for j in range(len(samples))],
                              len(samples) * BLOCK)
            for j in range(len(samples)):
                got = np.frombuffer(probe.read_range(j * size, size), dtype=np.uint8)
                parts = [gathered[src][j].cpu().numpy() for src in plan.sources(rank)]
                span = BLOCK * HEAD_DIM * 2                      # one head's bytes in a K or V span
                want = []
                for s_idx in range(2 * layers):                  # spans in layer-name order: k, v per layer
                    rows = [p[s_idx * span * (dst_heads // plan.groups):(s_idx + 1) * span * (dst_heads // plan.groups)]
                            .reshape(BLOCK, dst_heads // plan.groups, HEAD_DIM * 2) for p in parts]
                    want.append(np.concatenate(rows, axis=1).reshape(-1))
                ok &= bool(np.array_equal(got, np.concatenate(want)))
    flags = torch.tensor([1.0 if ok else 0.0], device=device)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    med = {key: statistics.median(r[key] for r in runs if key in r) for key in runs[-1]}
    worst = torch.tensor([med["total_s"], med.get("kernel_ms", 0.0), med["stage_s"]], dtype=torch.float64,
                         device=device)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    moved = plan.dst_tp * n * size
    result = {
        "workload": f"TP-{plan.src_tp} -> TP-{plan.dst_tp} regroup restore, qwen3-32b shape, 32768 tokens",
        "n_gpus": world, "blocks": n, "shard_bytes_per_rank": n * shard, "dest_bytes_per_rank": n * size,
        "total_ms": round(worst[0].item() * 1e3, 3), "regroup_kernel_ms": round(worst[1].item(), 3),
        "stage_ms": round(worst[2].item() * 1e3, 3),
        "regroup_kernel_gbs_per_dest_rank": round(n * size / (worst[1].item() / 1e3) / 1e9, 1),
        "box_restored_gbs": round(moved / worst[0].item() / 1e9, 2),
        "bit_exact_samples": bool(flags.item() == 1.0),
        "limit": "stage: every source rank's shard over the box's shared host link; kernel: peer reads over NVLink"}
    snapshot.close()
    plane.close()
    del plane, caches, noise
    release_device_memory()
    return result


def run_reshard(args, world, rank, device):
    """``--workload reshard``: the regroup alone, its line printed by rank 0."""
    import torch.distributed as dist
    result = measure_reshard(args, world, rank, device)
    if rank == 0:
        print(json.dumps(result), flush=True)
    dist.destroy_process_group()




def run_rotation(args, world, rank, device):
    """Benchmark configuration 4: 64 Qwen3-1.7B sessions saved and restored beside synthetic decode traffic.

    Session lengths are log-uniform in [512, 8192] tokens (seeded); blocks come
    from a shuffled free list (fragmented tables). Sessions 32..63 fork sessions
    0..31: their first 75% of blocks are copies of the parent's, so those blocks
    pack to the same bytes and the same content ids. All 64 are saved through the
    API (two save threads, digests on the GPU) and then restored into fresh blocks
    (one load thread), while a side stream keeps copying a 4 GiB buffer (HBM
    traffic standing in for decode). Reported: save/restore GB/s with and without
    the traffic, the traffic's GB/s with and without the data plane, and the dedup
    rate from the GPU digests beside the one from hashlib over the saved bytes.
    """
    import hashlib
    import threading
    import numpy as np
    import torch
    from kvsnap_b200.dataplane import PendingDigests, TorchBlockDataPlane
    layers, pool_blocks = 28, 32768
    rng = np.random.Generator(np.random.PCG64(args.seed + 44))
    lengths = np.exp(rng.uniform(np.log(512), np.log(8192), 64)).astype(int)
    for child in range(32, 64):                        # a fork is at least as long as 75% of its parent
        lengths[child] = max(lengths[child], int(lengths[child - 32]))
    free = [int(b) for b in rng.permutation(pool_blocks - 1) + 1]
    sessions = []
    for tokens in lengths:
        n = (int(tokens) + BLOCK - 1) // BLOCK
        sessions.append((int(tokens), [free.pop() for _ in range(n)]))
    caches = {}
    gen = torch.Generator(device=device)
    for i in range(layers):
        gen.manual_seed(args.seed * 1000 + 500 + i)
        t = torch.empty((2, pool_blocks, BLOCK, HEADS, HEAD_DIM), dtype=torch.bfloat16, device=device)
        t.normal_(generator=gen)
        caches[f"model.layers.{i}.self_attn.attn"] = t
    for child in range(32, 64):                        # forks copy 75% of the parent's full blocks
        parent_blocks = sessions[child - 32][1]
        shared = (len(parent_blocks) - 1) * 3 // 4
        src = torch.tensor(parent_blocks[:shared], device=device)
        dst = torch.tensor(sessions[child][1][:shared], device=device)
        for t in caches.values():
            t[:, dst] = t[:, src]
    total_blocks = sum(len(b) for _, b in sessions)
    size_guess = layers * 2 * BLOCK * HEADS * HEAD_DIM * 2
    plane = TorchBlockDataPlane(caches, BLOCK, total_blocks * size_guess + (512 << 20), ctas=args.ctas)
    plane.warm_up()
    size = plane.block_bytes
    snapshots = [[plane.pool.reserve(size) for _ in blocks] for _, blocks in sessions]
    restore_tables = [[free.pop() for _ in blocks] for _, blocks in sessions]

    decode_src = torch.empty(4 << 30, dtype=torch.uint8, device=device)
    decode_dst = torch.empty_like(decode_src)
    decode_stream = torch.cuda.Stream(device)
    stop = threading.Event()
    decoded = [0]

    def decode_loop():
        with torch.cuda.stream(decode_stream):
            while not stop.is_set():
                decode_dst.copy_(decode_src, non_blocking=True)
                decoded[0] += 1
                decode_stream.synchronize()

    def decode_rate(seconds):
        decoded[0] = 0
        stop.clear()
        thread = threading.Thread(target=decode_loop)
        t0 = time.perf_counter()
        thread.start()
        time.sleep(seconds)
        stop.set()
        thread.join()
        return 2 * decoded[0] * decode_src.numel() / (time.perf_counter() - t0) / 1e9

    def rotate(with_decode):
        digests = [None] * len(sessions)
        savers, loader = ThreadPoolExecutor(max_workers=2), ThreadPoolExecutor(max_workers=1)
        thread = None
        if with_decode:
            decoded[0] = 0
            stop.clear()
            thread = threading.Thread(target=decode_loop)
            thread.start()
        torch.cuda.synchronize()
        t0 = time.perf_counter()

        def save(i):
            # The save returns once its blocks are in pinned memory; its digests follow.
            pending = PendingDigests()
            tokens, blocks = sessions[i]
            plane.save_gather(blocks, [(a, 0) for a in snapshots[i]], tokens, digests=pending)
            digests[i] = pending

        list(savers.map(save, range(len(sessions))))
        digests = [d.result() for d in digests]
        t_saved = time.perf_counter()
        list(loader.map(lambda i: plane.load_scatter(restore_tables[i], [(a, 0) for a in snapshots[i]]),
                        range(len(sessions))))
        t1 = time.perf_counter()
        decode_gbs = None
        if thread is not None:
            stop.set()
            thread.join()
            decode_gbs = 2 * decoded[0] * decode_src.numel() / (time.perf_counter() - t0) / 1e9
        savers.shutdown()
        loader.shutdown()
        return digests, t_saved - t0, t1 - t_saved, decode_gbs

    rotate(False)                                        # warm
    digests, save_s, restore_s, _ = rotate(False)
    _, save_s_busy, restore_s_busy, decode_busy = rotate(True)
    decode_alone = decode_rate(2.0)
    ids = [d[0] for ds in digests for d in ds]
    gpu_dedup = 1 - len(set(ids)) / len(ids)
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as hashers:
        host_ids = list(hashers.map(lambda a: hashlib.sha256(a.read()).hexdigest(),
                                    [a for owned in snapshots for a in owned]))
    host_dedup = 1 - len(set(host_ids)) / len(host_ids)
    moved = total_blocks * size
    if rank == 0:
        print(json.dumps({
            "workload": "64-session rotation, qwen3-1.7b shape (BASELINE config 4)",
            "sessions": len(sessions), "blocks": total_blocks, "bytes_each_way": moved,
            "save_gbs": round(moved / save_s / 1e9, 2), "restore_gbs": round(moved / restore_s / 1e9, 2),
            "save_gbs_beside_decode": round(moved / save_s_busy / 1e9, 2),
            "restore_gbs_beside_decode": round(moved / restore_s_busy / 1e9, 2),
            "decode_gbs_alone": round(decode_alone, 1), "decode_gbs_beside_data_plane": round(decode_busy, 1),
            "dedup_rate_gpu": round(gpu_dedup, 6), "dedup_rate_hashlib": round(host_dedup, 6),
            "dedup_match": gpu_dedup == host_dedup and ids == host_ids}), flush=True)
    for owned in snapshots:
        for a in owned:
            a.close()
    plane.close()


def explore_phases(plane, engine, save_ids, restore_ids, link):
    """Each phase alone, and the restore kernel over a sweep of CTA counts and both modes."""
    import torch
    lib, n, size = engine.lib, engine.n, engine.size
    nspans = len(plane.layers)
    out = {"link": link}

    def timed(fn, reps=5):
        fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(engine.copy)
        for _ in range(reps):
            fn()
        e.record(engine.copy)
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps

    for ctas in (0, 16, 32, 64, 148, 296, 592):
        def restore():
            lib.kvsnap_dp_scatter(engine.spans.data_ptr(), nspans, size, engine.pinned_addrs[0].data_ptr(),
                                  engine.restore_ids.data_ptr(), n, 0, 0, 0, engine.status.data_ptr(), 16, ctas,
                                  engine.copy.cuda_stream)

        def restore_crc():
            lib.kvsnap_dp_scatter(engine.spans.data_ptr(), nspans, size, engine.pinned_addrs[0].data_ptr(),
                                  engine.restore_ids.data_ptr(), n, engine.crc_restore.data_ptr(), 0, 0,
                                  engine.status.data_ptr(), 16, ctas, engine.copy.cuda_stream)

        def gather():
            lib.kvsnap_dp_gather(engine.spans.data_ptr(), nspans, size, engine.save_ids.data_ptr(),
                                 engine.stage_addrs[0].data_ptr(), n, 0, engine.crc[0].data_ptr(), engine.status.data_ptr(),
                                 16, ctas, engine.copy.cuda_stream)

        def gather_nocrc():
            lib.kvsnap_dp_gather(engine.spans.data_ptr(), nspans, size, engine.save_ids.data_ptr(),
                                 engine.stage_addrs[0].data_ptr(), n, 0, 0, engine.status.data_ptr(), 16, ctas,
                                 engine.copy.cuda_stream)

        def scatter_hbm():
            lib.kvsnap_dp_scatter(engine.spans.data_ptr(), nspans, size, engine.stage_addrs[0].data_ptr(),
                                  engine.restore_ids.data_ptr(), n, engine.crc_restore.data_ptr(), 0, 0,
                                  engine.status.data_ptr(), 16, ctas, engine.copy.cuda_stream)

        def scatter_lc():
            lib.kvsnap_dp_scatter(engine.spans.data_ptr(), nspans, size, engine.stage_addrs[0].data_ptr(),
                                  engine.restore_ids.data_ptr(), n, engine.crc_restore.data_ptr(), 0, 0,
                                  engine.status.data_ptr(), 16 | plane._hbm, ctas, engine.copy.cuda_stream)

        def gather_lc():
            lib.kvsnap_dp_gather(engine.spans.data_ptr(), nspans, size, engine.save_ids.data_ptr(),
                                 engine.stage_addrs[0].data_ptr(), n, 0, engine.crc[0].data_ptr(), engine.status.data_ptr(),
                                 16 | plane._hbm, ctas, engine.copy.cuda_stream)

        def gather_lc_nocrc():
            lib.kvsnap_dp_gather(engine.spans.data_ptr(), nspans, size, engine.save_ids.data_ptr(),
                                 engine.stage_addrs[0].data_ptr(), n, 0, 0, engine.status.data_ptr(),
                                 16 | plane._hbm, ctas, engine.copy.cuda_stream)

        def gather_direct():
            lib.kvsnap_dp_gather(engine.spans.data_ptr(), nspans, size, engine.save_ids.data_ptr(),
                                 engine.pinned_addrs[0].data_ptr(), n, 0, engine.crc[0].data_ptr(),
                                 engine.status.data_ptr(), 16, ctas, engine.copy.cuda_stream)

        row = {}
        for name, fn, nbytes in (("restore_direct", restore, size * n), ("restore_direct_crc", restore_crc, size * n),
                                 ("gather_hbm_crc", gather, 2 * size * n), ("gather_hbm", gather_nocrc, 2 * size * n),
                                 ("scatter_hbm_crc", scatter_hbm, 2 * size * n),
                                 ("scatter_lc_crc", scatter_lc, 2 * size * n), ("gather_lc_crc", gather_lc, 2 * size * n),
                                 ("gather_lc", gather_lc_nocrc, 2 * size * n),
                                 ("gather_direct_crc", gather_direct, size * n)):
            ms = timed(fn)
            row[name] = {"ms": round(ms, 3), "gbs": round(nbytes / (ms / 1e3) / 1e9, 2)}
        out[f"ctas={ctas}"] = row

    def sha():
        lib.kvsnap_dp_sha256(engine.stage_addrs[0].data_ptr(), n, size, engine.digest[0].data_ptr(), engine.copy.cuda_stream)

    def d2h():
        lib.kvsnap_pool_copy(engine.handle, engine.snapshot[0].ident, 0, engine.stage[0].data_ptr(), n * size, 1,
                             engine.copy.cuda_stream)

    def h2d():
        lib.kvsnap_pool_copy(engine.handle, engine.snapshot[0].ident, 0, engine.stage[0].data_ptr(), n * size, 0, 0)

    for name, fn in (("sha256", sha), ("d2h_pool", d2h), ("h2d_pool", h2d)):
        ms = timed(fn, reps=3)
        out[name] = {"ms": round(ms, 3), "gbs": round(n * size / (ms / 1e3) / 1e9, 2)}

    # Both directions of the host link at once: device-to-host by the copy engine on the copy stream,
    # host-to-device either by a second copy engine or by the scatter kernel on the load stream.
    dev_in = torch.empty(n * size, dtype=torch.uint8, device=engine.stage[0].device)
    pinned_in = torch.empty(n * size, dtype=torch.uint8, pin_memory=True)

    def duplex(kernel):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(engine.copy)
        engine.load.wait_event(start)
        for _ in range(3):
            d2h()
            if kernel:
                lib.kvsnap_dp_scatter(engine.spans.data_ptr(), nspans, size, engine.pinned_addrs[1].data_ptr(),
                                      engine.restore_ids.data_ptr(), n, 0, 0, 0, engine.status.data_ptr(), 16,
                                      plane.host_ctas, engine.load.cuda_stream)
            else:
                with torch.cuda.stream(engine.load):
                    dev_in.copy_(pinned_in, non_blocking=True)
        done = torch.cuda.Event()
        done.record(engine.load)
        engine.copy.wait_event(done)
        end.record(engine.copy)
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / 3
        return {"ms_per_pair": round(ms, 3), "gbs_both": round(2 * n * size / (ms / 1e3) / 1e9, 2)}

    out["duplex_dma"] = duplex(False)
    out["duplex_dma_kernel"] = duplex(True)
    return out


if __name__ == "__main__":
    main()
