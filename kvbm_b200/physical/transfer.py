"""Transfer planning and execution between registered KV layouts.

``TransferManager`` registers layouts of every tier (G1 device, G2 pinned
host, G3 disk, peer G1 pools mapped over NVLink), exports/imports their
metadata between processes, and executes block transfers by handle:

* device/pinned/peer pairs run on SM kernels (``ops.kv_ops``): one fused
  launch per transfer, with any layout transform, head slice or fp8 cast
  folded in; plain whole-block copies between identical fully contiguous
  layouts use the split-by-bytes pair copy; the copy engine
  (``cudaMemcpyAsync`` per contiguous region) is kept as an explicit option
  and as the measured baseline;
* pinned <-> disk run on the native ``DiskPool`` thread pool (pread/pwrite);
* device <-> disk go through a pinned bounce layout (two hops).

Completion is a :class:`TransferCompleteNotification` (CUDA event or I/O
future). Streams come from a pool of 4 H2D + 4 D2H + 1 D2D streams.

Parity: crates/kvbm-physical/src/manager/mod.rs:49-490 (TransferManager:
register_layout, export/import_metadata, execute_transfer,
execute_transfer_selection), transfer/strategy.rs:16-230 (strategy matrix,
two-hop plans), transfer/capabilities.rs:53-140, transfer/options.rs:30-80,
transfer/context.rs:333-342 (4+4 streams), notifications/* (completion).
"""

from __future__ import annotations

import collections
import concurrent.futures as cf
import dataclasses
import enum
import itertools
import logging
import threading
import time
from dataclasses import dataclass, field

import torch

from .. import _core_native as core
from ..ops import kv_ops
from .layout import KvBlockLayout, KvLayout, LayoutConfig, LayoutDescriptor
from .plan import PreparedPlanCache, lower, plan_copy

log = logging.getLogger(__name__)


class StorageKind(str, enum.Enum):
    DEVICE = "device"   # G1
    PINNED = "pinned"   # G2
    SYSTEM = "system"
    DISK = "disk"       # G3
    OBJECT = "object"   # G4
    PEER = "peer"       # another GPU's G1, mapped over NVLink


class TransferStrategy(str, enum.Enum):
    MEMCPY = "memcpy"
    CUDA_ASYNC_H2D = "cuda_async_h2d"
    CUDA_ASYNC_D2H = "cuda_async_d2h"
    CUDA_ASYNC_D2D = "cuda_async_d2d"
    KERNEL_H2D = "kernel_h2d"
    KERNEL_D2H = "kernel_d2h"
    KERNEL_D2D = "kernel_d2d"
    KERNEL_P2P = "kernel_p2p"
    DISK_READ = "disk_read"
    DISK_WRITE = "disk_write"
    INVALID = "invalid"


@dataclass(frozen=True)
class TransferPlan:
    first: TransferStrategy
    bounce: StorageKind | None = None
    second: TransferStrategy | None = None

    @property
    def is_two_hop(self) -> bool:
        return self.second is not None


@dataclass
class TransferCapabilities:
    """Feature switches for direct paths (all off by default, as upstream)."""

    allow_gds: bool = False          # device <-> disk without a host bounce
    allow_gpu_rdma: bool = False     # device -> remote without a host bounce
    cuda_graph_replay: bool = False
    startup_benchmark: bool = False
    prefer_copy_engine: bool = False  # use cudaMemcpyAsync instead of SM kernels


def select_strategy(src: StorageKind, dst: StorageKind, caps: TransferCapabilities | None = None) -> TransferPlan:
    """Direct/two-hop plan for a local (or peer-mapped) src -> dst pair."""
    caps = caps or TransferCapabilities()
    S, D = src, dst
    K = StorageKind
    ce = caps.prefer_copy_engine
    host = (K.PINNED, K.SYSTEM)
    if S in host and D in host:
        return TransferPlan(TransferStrategy.MEMCPY)
    if S in host and D == K.DEVICE:
        return TransferPlan(TransferStrategy.CUDA_ASYNC_H2D if ce else TransferStrategy.KERNEL_H2D)
    if S == K.DEVICE and D in host:
        return TransferPlan(TransferStrategy.CUDA_ASYNC_D2H if ce else TransferStrategy.KERNEL_D2H)
    if S == K.DEVICE and D == K.DEVICE:
        return TransferPlan(TransferStrategy.CUDA_ASYNC_D2D if ce else TransferStrategy.KERNEL_D2D)
    if S == K.DEVICE and D == K.PEER:
        return TransferPlan(TransferStrategy.KERNEL_P2P)
    if S == K.PINNED and D == K.DISK:
        return TransferPlan(TransferStrategy.DISK_WRITE)
    if S == K.DISK and D == K.PINNED:
        return TransferPlan(TransferStrategy.DISK_READ)
    if S == K.DEVICE and D == K.DISK:
        if caps.allow_gds:
            return TransferPlan(TransferStrategy.DISK_WRITE)
        return TransferPlan(TransferStrategy.KERNEL_D2H, K.PINNED, TransferStrategy.DISK_WRITE)
    if S == K.DISK and D == K.DEVICE:
        if caps.allow_gds:
            return TransferPlan(TransferStrategy.DISK_READ)
        return TransferPlan(TransferStrategy.DISK_READ, K.PINNED, TransferStrategy.KERNEL_H2D)
    return TransferPlan(TransferStrategy.INVALID)


@dataclass
class TransferOptions:
    layer_range: tuple[int, int] | None = None      # [begin, end)
    head_range: tuple[int, int, int] | None = None  # (src_offset, dst_offset, num_heads)
    engine: str = "auto"                            # auto | tile | tma | pairs | ce
    stream: torch.cuda.Stream | None = None         # caller-owned stream: no event recorded
    max_ctas: int = 0
    bounce: "PhysicalLayout | None" = None


class TransferCompleteNotification:
    """Completion of one transfer: a CUDA event, an I/O future, or already done."""

    def __init__(self, event: torch.cuda.Event | None = None, future: cf.Future | None = None,
                 parts: list["TransferCompleteNotification"] | None = None):
        self._event, self._future, self._parts = event, future, parts or []

    @classmethod
    def ready(cls) -> "TransferCompleteNotification":
        return cls()

    @classmethod
    def aggregate(cls, notes: list["TransferCompleteNotification"]) -> "TransferCompleteNotification":
        return cls(parts=list(notes))

    def is_complete(self) -> bool:
        if self._event is not None and not self._event.query():
            return False
        if self._future is not None and not self._future.done():
            return False
        return all(p.is_complete() for p in self._parts)

    def wait(self, timeout: float | None = None) -> None:
        deadline = None if timeout is None else time.monotonic() + timeout
        for p in self._parts:
            p.wait(None if deadline is None else max(0.0, deadline - time.monotonic()))
        if self._future is not None:
            self._future.result(timeout=None if deadline is None else max(0.0, deadline - time.monotonic()))
        if self._event is not None:
            if deadline is None:
                self._event.synchronize()
            else:
                while not self._event.query():
                    if time.monotonic() > deadline:
                        raise TimeoutError("transfer did not complete in time")
                    time.sleep(50e-6)

    def stream_wait(self, stream: torch.cuda.Stream) -> None:
        """Make ``stream`` wait for this transfer without blocking the host."""
        for p in self._parts:
            p.stream_wait(stream)
        if self._future is not None:
            self._future.result()
        if self._event is not None:
            stream.wait_event(self._event)


class DiskLayout:
    """G3 pool: ``num_blocks`` block-contiguous slots in one file."""

    def __init__(self, config: LayoutConfig, path: str, direct: bool = True, persistent: bool = False,
                 threads: int = 4, block_layout: KvBlockLayout = KvBlockLayout.OPERATIONAL_NHD):
        self.config = config
        self.block_layout = block_layout
        self.path, self.direct = path, direct
        self.pool = core.DiskPool(path, config.num_blocks, config.bytes_per_block, direct, persistent, threads)
        self._gds = None

    def gds_file(self):
        """The file opened for cuFile I/O (GPUDirect Storage), on first use."""
        if self._gds is None:
            from .gds import GdsFile

            fd = self.pool.fd_direct if self.pool.fd_direct >= 0 else self.pool.fd  # the file may be unlinked
            self._gds = GdsFile(self.path, self.config.bytes_per_block, direct=self.direct, fd=fd)
        return self._gds


@dataclass
class PhysicalLayout:
    kind: StorageKind
    layout: KvLayout | DiskLayout

    @property
    def config(self) -> LayoutConfig:
        return self.layout.config

    @classmethod
    def of(cls, layout: KvLayout | DiskLayout) -> "PhysicalLayout":
        if isinstance(layout, DiskLayout):
            return cls(StorageKind.DISK, layout)
        kind = {"device": StorageKind.DEVICE, "pinned": StorageKind.PINNED, "peer": StorageKind.PEER}[layout.location]
        return cls(kind, layout)


@dataclass
class SerializedLayouts:
    worker_id: int
    layouts: dict[int, dict] = field(default_factory=dict)  # layout_id -> LayoutDescriptor dict


class TransferManager:
    """Layout registry + transfer executor for one worker (one GPU)."""

    def __init__(self, worker_id: int = 0, device: int | None = None, capabilities: TransferCapabilities | None = None,
                 num_h2d_streams: int = 4, num_d2h_streams: int = 4, io_threads: int = 4):
        self.worker_id = worker_id
        self.device = device
        self.caps = capabilities or TransferCapabilities()
        if self.caps.allow_gds:
            from .gds import gds_available, gds_status

            if not gds_available():
                # cuFile cannot run here: device <-> disk goes through the pinned bounce instead
                log.warning("GDS requested but cuFile is unavailable (status %d); using the two-hop path",
                            gds_status())
                self.caps = dataclasses.replace(self.caps, allow_gds=False)
        self._layouts: dict[int, PhysicalLayout] = {}
        self._ids = itertools.count(1)
        self._lock = threading.Lock()
        self._h2d: list[torch.cuda.Stream] = []
        self._d2h: list[torch.cuda.Stream] = []
        self._d2d: torch.cuda.Stream | None = None
        self._n_h2d, self._n_d2h = num_h2d_streams, num_d2h_streams
        self._rr = itertools.count()
        self._io = cf.ThreadPoolExecutor(max_workers=io_threads, thread_name_prefix="kvbm-io")
        self._bounce: PhysicalLayout | None = None
        self._plans = PreparedPlanCache()
        self._ce_graphs: collections.OrderedDict[tuple, torch.cuda.CUDAGraph] = collections.OrderedDict()
        self._bench = None  # StartupBenchmark, created by calibrate() when caps.startup_benchmark is on
        self.stats = {"transfers": 0, "bytes": 0, "failures": 0}

    # ------------------------------------------------------------ registry
    def register_layout(self, layout: KvLayout | DiskLayout | PhysicalLayout) -> int:
        pl = layout if isinstance(layout, PhysicalLayout) else PhysicalLayout.of(layout)
        with self._lock:
            lid = next(self._ids)
            self._layouts[lid] = pl
        return (self.worker_id << 64) | lid

    def layout(self, handle: int) -> PhysicalLayout:
        try:
            return self._layouts[handle & ((1 << 64) - 1)]
        except KeyError:
            raise KeyError(f"unknown layout handle {handle:#x}") from None

    def set_bounce(self, layout: KvLayout) -> None:
        """Pinned layout used as the staging hop for device <-> disk transfers."""
        self._bounce = PhysicalLayout.of(layout)

    def export_metadata(self) -> SerializedLayouts:
        out = SerializedLayouts(self.worker_id)
        for lid, pl in self._layouts.items():
            if pl.kind == StorageKind.DEVICE and isinstance(pl.layout.backing, object):
                try:
                    out.layouts[lid] = pl.layout.descriptor().to_dict()
                except ValueError:
                    continue
        return out

    def import_metadata(self, meta: SerializedLayouts) -> dict[int, int]:
        """Map a peer's exported device pools; returns remote handle -> local handle."""
        mapping = {}
        for lid, d in meta.layouts.items():
            lay = KvLayout.from_descriptor(LayoutDescriptor.from_dict(d), device=self.device)
            mapping[(meta.worker_id << 64) | lid] = self.register_layout(PhysicalLayout(StorageKind.PEER, lay))
        return mapping

    # ------------------------------------------------------------- streams
    def _stream(self, kind: str) -> torch.cuda.Stream:
        if not self._h2d:
            self._h2d = [torch.cuda.Stream() for _ in range(self._n_h2d)]
            self._d2h = [torch.cuda.Stream() for _ in range(self._n_d2h)]
            self._d2d = torch.cuda.Stream()
        i = next(self._rr)
        if kind == "h2d":
            return self._h2d[i % len(self._h2d)]
        if kind == "d2h":
            return self._d2h[i % len(self._d2h)]
        return self._d2d

    # ------------------------------------------------------------ execute
    @staticmethod
    def _validate(ids, n: int, what: str) -> list[int]:
        ids = [int(i) for i in (ids.tolist() if isinstance(ids, torch.Tensor) else ids)]
        for i in ids:
            if i < 0 or i >= n:
                raise IndexError(f"{what} block id {i} out of range [0, {n})")
        return ids

    def execute_transfer(self, src_handle: int, src_ids, dst_handle: int, dst_ids,
                         options: TransferOptions | None = None) -> TransferCompleteNotification:
        opts = options or TransferOptions()
        src, dst = self.layout(src_handle), self.layout(dst_handle)
        s_ids = self._validate(src_ids, src.config.num_blocks, "source")
        d_ids = self._validate(dst_ids, dst.config.num_blocks, "destination")
        if len(s_ids) != len(d_ids):
            raise ValueError("source and destination id lists differ in length")
        if not s_ids:
            return TransferCompleteNotification.ready()
        plan = select_strategy(src.kind, dst.kind, self.caps)
        if plan.first == TransferStrategy.INVALID:
            raise ValueError(f"no transfer path from {src.kind.value} to {dst.kind.value}")
        try:
            if plan.is_two_hop:
                note = self._two_hop(src, s_ids, dst, d_ids, plan, opts)
            else:
                note = self._direct(src, s_ids, dst, d_ids, plan.first, opts)
        except Exception:
            self.stats["failures"] += 1
            raise
        self.stats["transfers"] += 1
        self.stats["bytes"] += len(s_ids) * src.config.bytes_per_block
        return note

    def execute_transfer_selection(self, src_handle: int, src_ids, dst_handle: int, dst_ids,
                                   layer_range: tuple[int, int] | None = None,
                                   head_range: tuple[int, int, int] | None = None,
                                   options: TransferOptions | None = None) -> TransferCompleteNotification:
        """Axis-sliced transfer: a layer range and/or a KV-head slice (TP resharding)."""
        opts = options or TransferOptions()
        opts.layer_range = layer_range or opts.layer_range
        opts.head_range = head_range or opts.head_range
        return self.execute_transfer(src_handle, src_ids, dst_handle, dst_ids, opts)

    def _pick_engine(self, src: KvLayout, dst: KvLayout, opts: TransferOptions, s_ids=(), d_ids=()) -> str:
        """Plan (``plan.plan_copy``) and lower (``plan.lower``) the transfer; the choice is
        memoised per layout pair and ranges (it does not depend on the block ids)."""
        key = PreparedPlanCache.key(src, dst, opts.layer_range, opts.head_range, opts.engine)
        hit = self._plans.get(key)
        if hit is not None:
            return hit.engine
        plan = plan_copy(src, s_ids, dst, d_ids, opts.layer_range, opts.head_range)
        bench = None
        if self.caps.startup_benchmark and self._bench is not None:
            bench = self._bench.lookup(src, dst)
        low = lower(plan, src, dst, prefer_copy_engine=self.caps.prefer_copy_engine, engine=opts.engine,
                    bench_choice=bench)
        if bench is not None or not self.caps.startup_benchmark:
            self._plans.put(key, low)  # a pair not yet calibrated may get a benchmark result later
        return low.engine

    def calibrate(self, src_handle: int, dst_handle: int) -> str:
        """Run (or load from the cache) the startup benchmark for a layout pair; returns the chosen engine."""
        from .verify import StartupBenchmark

        if self._bench is None:
            self._bench = StartupBenchmark()
        return self._bench.run(self, src_handle, dst_handle)

    def _direct(self, src: PhysicalLayout, s_ids, dst: PhysicalLayout, d_ids, strat: TransferStrategy,
                opts: TransferOptions) -> TransferCompleteNotification:
        if strat in (TransferStrategy.DISK_WRITE, TransferStrategy.DISK_READ):
            return self._disk(src, s_ids, dst, d_ids, strat)
        if strat == TransferStrategy.MEMCPY:
            return self._host_copy(src.layout, s_ids, dst.layout, d_ids, opts)
        kind = "h2d" if strat in (TransferStrategy.KERNEL_H2D, TransferStrategy.CUDA_ASYNC_H2D) else (
            "d2h" if strat in (TransferStrategy.KERNEL_D2H, TransferStrategy.CUDA_ASYNC_D2H) else "d2d")
        stream = opts.stream or self._stream(kind)
        a, b = src.layout, dst.layout
        engine = "ce" if strat.value.startswith("cuda_async") else self._pick_engine(a, b, opts, s_ids, d_ids)
        lb, le = opts.layer_range or (0, a.config.num_layers)
        with torch.cuda.stream(stream):
            if engine == "ce":
                sp, dp, size = self._regions(a, s_ids, b, d_ids, lb, le)
                if self.caps.cuda_graph_replay:
                    self._replay_ce(sp, dp, size, stream)
                else:
                    kv_ops.memcpy_pairs_ce(sp, dp, size, stream=stream)
            elif engine == "pairs":
                sp = [a.layer_base(0) + i * a.block_stride for i in s_ids]
                dp = [b.layer_base(0) + i * b.block_stride for i in d_ids]
                kv_ops.copy_pairs(sp, dp, a.config.bytes_per_block, max_ctas=opts.max_ctas, stream=stream)
            else:
                hr = opts.head_range
                sid = kv_ops.upload(torch.tensor(s_ids, dtype=torch.int32), stream.device, stream)
                did = kv_ops.upload(torch.tensor(d_ids, dtype=torch.int32), stream.device, stream)
                # an engine the manager chose itself may fall back; one the caller forced may not
                run = "auto" if (engine == "tma" and opts.engine == "auto") else engine
                self.last_engine = kv_ops.kv_transfer(a, sid, b, did, layer_begin=lb, num_layers=le - lb,
                                                      src_head_offset=hr[0] if hr else 0,
                                                      dst_head_offset=hr[1] if hr else 0,
                                                      num_heads=hr[2] if hr else None, engine=run,
                                                      max_ctas=opts.max_ctas, stream=stream)
            if opts.stream is not None:
                return TransferCompleteNotification.ready()
            ev = torch.cuda.Event()
            ev.record(stream)
        return TransferCompleteNotification(event=ev)

    def _replay_ce(self, sp: list[int], dp: list[int], size: int, stream: torch.cuda.Stream) -> None:
        """Copy-engine regions as a replayed CUDA graph of memcpy nodes: captured the first
        time a region list is seen, replayed on ``stream`` afterwards (LRU of 64 graphs)."""
        key = (tuple(sp), tuple(dp), size)
        g = self._ce_graphs.get(key)
        if g is None:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                kv_ops.memcpy_pairs_ce(sp, dp, size, stream=torch.cuda.current_stream())
            self._ce_graphs[key] = g
            self.stats["graph_captures"] = self.stats.get("graph_captures", 0) + 1
            while len(self._ce_graphs) > 64:
                self._ce_graphs.popitem(last=False)
        else:
            self._ce_graphs.move_to_end(key)
        with torch.cuda.stream(stream):
            g.replay()
        self.stats["graph_replays"] = self.stats.get("graph_replays", 0) + 1

    @staticmethod
    def _regions(a: KvLayout, s_ids, b: KvLayout, d_ids, lb: int, le: int):
        """Contiguous (src, dst, size) regions for the copy-engine path."""
        if (a.kind == b.kind == "fully_contiguous" and a.block_layout == b.block_layout and (lb, le) ==
                (0, a.config.num_layers) and a.block_layout != KvBlockLayout.UNIVERSAL):
            return ([a.layer_base(0) + i * a.block_stride for i in s_ids],
                    [b.layer_base(0) + i * b.block_stride for i in d_ids], a.config.bytes_per_block)
        if a.block_layout != b.block_layout:
            raise ValueError("the copy engine cannot transform layouts; use an SM kernel engine")
        sp, dp = [], []
        for si, di in zip(s_ids, d_ids):
            for l in range(lb, le):
                for o in range(a.config.outer_dim):
                    sp.append(a.memory_region(si, l, o)[0])
                    dp.append(b.memory_region(di, l, o)[0])
        return sp, dp, a.config.bytes_per_chunk

    def _host_copy(self, a: KvLayout, s_ids, b: KvLayout, d_ids, opts) -> TransferCompleteNotification:
        def run():
            data = a.gather_blocks(s_ids)
            b.scatter_blocks(d_ids, data)
        return TransferCompleteNotification(future=self._io.submit(run))

    def _disk(self, src: PhysicalLayout, s_ids, dst: PhysicalLayout, d_ids, strat) -> TransferCompleteNotification:
        if strat == TransferStrategy.DISK_WRITE:
            host, disk, h_ids, k_ids = src.layout, dst.layout, s_ids, d_ids
        else:
            host, disk, h_ids, k_ids = dst.layout, src.layout, d_ids, s_ids
        if not isinstance(host, KvLayout) or host.kind != "fully_contiguous":
            raise ValueError("disk transfers need a fully contiguous layout on the other side")
        if host.block_stride != disk.config.bytes_per_block:
            raise ValueError("memory and disk block sizes differ")
        if host.location == "device":
            # GPUDirect Storage: cuFile moves the blocks between HBM and the file
            if not self.caps.allow_gds:
                raise ValueError("device <-> disk needs allow_gds (or the two-hop plan)")
            gds = disk.gds_file()
            write = strat == TransferStrategy.DISK_WRITE
            base = host.layer_base(0)
            if self.device is not None:
                torch.cuda.current_stream(self.device).synchronize()  # the blocks' producers are done
            else:
                torch.cuda.current_stream().synchronize()
            return TransferCompleteNotification(future=self._io.submit(
                gds.transfer, write, base, host.block_stride, list(h_ids), list(k_ids)))
        ptrs = [host.layer_base(0) + i * host.block_stride for i in h_ids]
        fn = disk.pool.write if strat == TransferStrategy.DISK_WRITE else disk.pool.read
        return TransferCompleteNotification(future=self._io.submit(fn, list(k_ids), ptrs))

    def _two_hop(self, src, s_ids, dst, d_ids, plan: TransferPlan, opts) -> TransferCompleteNotification:
        bounce = opts.bounce or self._bounce
        if bounce is None:
            raise ValueError("two-hop transfer needs a bounce layout (TransferManager.set_bounce)")
        cap = bounce.config.num_blocks
        note = None
        for i in range(0, len(s_ids), cap):  # transfers larger than the bounce go through it in chunks
            cs, cd = s_ids[i:i + cap], d_ids[i:i + cap]
            b_ids = list(range(len(cs)))
            if note is not None:
                note.wait()  # the previous chunk's second hop has drained the bounce
            first = self._direct(src, cs, bounce, b_ids, plan.first, TransferOptions(engine=opts.engine))
            first.wait()
            note = self._direct(bounce, b_ids, dst, cd, plan.second, TransferOptions(engine=opts.engine))
        return note

    def close(self) -> None:
        self._io.shutdown(wait=True)
