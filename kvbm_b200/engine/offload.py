"""Offload pipelines: G1 -> G2, G2 -> G3 and G2 -> G4, with policies,
preconditions, batching and cancellation.

A pipeline is one worker thread that moves *containers* (one per enqueue,
typically one request's newly completed blocks) through four stages:

1. policy evaluation - filters drop blocks the destination does not need
   (already present there, not frequent enough, already in the object store);
2. precondition - wait until the source data is final (e.g. the CUDA event
   recorded after the forward pass that wrote the G1 blocks);
3. batching - items are grouped up to ``max_batch`` and flushed when
   ``min_batch`` is reached or ``flush_ms`` passes;
4. execution - destination blocks are allocated, the transfer runs, and the
   blocks are registered in the destination tier under their sequence hashes.

A container can be cancelled until its blocks are registered; after that the
offload is final. G2 registrations can chain automatically into G2 -> G3.

Parity: crates/kvbm-engine/src/tiering/offload/{engine.rs:78-123 OffloadEngine,
pipeline.rs (PolicyEvaluator -> PreconditionAwaiter -> Batcher ->
TransferExecutor), policy.rs:277-893 (PresenceFilter, PresenceAndLFUFilter,
ObjectPresenceFilter, ObjectLockPresenceFilter, AllOf, AnyOf, PassAll),
batch.rs, queue.rs, cancel.rs, handle.rs}; defaults from docs/offload.md:88-99
(max_batch 64, min 8, flush 10 ms, policy timeout 100 ms, concurrency 1).
"""

from __future__ import annotations

import enum
import queue
import threading
import time
from dataclasses import dataclass
from typing import Callable, Sequence

from ..logical.manager import BlockManager, ImmutableBlock
from ..utils.config import PipelineConfig
from ..utils.tracing import audit, nvtx_range


@dataclass
class OffloadItem:
    seq_hash: int
    src_block_id: int
    src_ref: ImmutableBlock | None = None  # keeps the source block alive while queued


class OffloadState(str, enum.Enum):
    QUEUED = "queued"
    RUNNING = "running"
    DONE = "done"
    CANCELLED = "cancelled"
    FAILED = "failed"


class OffloadHandle:
    """One enqueued container; cancellable until its blocks are registered."""

    def __init__(self, items: list[OffloadItem], precondition: Callable[[], bool] | None):
        self.items = items
        self.precondition = precondition
        self.state = OffloadState.QUEUED
        self.registered: list[ImmutableBlock] = []
        self.skipped: list[int] = []
        self.error: BaseException | None = None
        self._done = threading.Event()
        self._lock = threading.Lock()
        self._cancel = False

    def cancel(self) -> bool:
        """Request cancellation; returns False if the offload already became final."""
        with self._lock:
            if self.state in (OffloadState.DONE, OffloadState.FAILED):
                return False
            self._cancel = True
            if self.state == OffloadState.QUEUED:
                self._finish(OffloadState.CANCELLED)
            return True

    @property
    def cancelled(self) -> bool:
        return self._cancel

    def _finish(self, st: OffloadState) -> None:
        self.state = st
        for it in self.items:
            it.src_ref = None
        self._done.set()

    def wait(self, timeout: float | None = None) -> OffloadState:
        if not self._done.wait(timeout):
            raise TimeoutError("offload did not finish in time")
        return self.state

    def done(self) -> bool:
        return self._done.is_set()


# ------------------------------------------------------------------ policies
class OffloadPolicy:
    def keep(self, item: OffloadItem) -> bool:  # pragma: no cover - interface
        raise NotImplementedError

    def filter(self, items: Sequence[OffloadItem]) -> list[OffloadItem]:
        return [i for i in items if self.keep(i)]


class PassAll(OffloadPolicy):
    def keep(self, item):
        return True


class PresenceFilter(OffloadPolicy):
    """Drop blocks the destination tier already holds."""

    def __init__(self, dst: BlockManager):
        self.dst = dst

    def keep(self, item):
        return not self.dst.registry.is_present(item.seq_hash, int(self.dst.tier))


class PresenceAndLFUFilter(OffloadPolicy):
    """Presence filter plus a minimum TinyLFU access count."""

    def __init__(self, dst: BlockManager, min_frequency: int = 2):
        self.presence = PresenceFilter(dst)
        self.dst, self.min_frequency = dst, min_frequency

    def keep(self, item):
        return self.presence.keep(item) and self.dst.registry.frequency(item.seq_hash) >= self.min_frequency


class ObjectPresenceFilter(OffloadPolicy):
    """Drop blocks whose key already exists in the object store."""

    def __init__(self, store, rank: int = 0):
        self.store, self.rank = store, rank

    def keep(self, item):
        return not self.store.has(self.store.key(item.seq_hash, self.rank))


class ObjectLockPresenceFilter(ObjectPresenceFilter):
    """Object presence + a conditional-put lock so one writer uploads a block."""

    def keep(self, item):
        key = self.store.key(item.seq_hash, self.rank)
        return not self.store.has(key) and self.store.try_lock(key)


class AllOf(OffloadPolicy):
    def __init__(self, *policies):
        self.policies = policies

    def keep(self, item):
        return all(p.keep(item) for p in self.policies)


class AnyOf(OffloadPolicy):
    def __init__(self, *policies):
        self.policies = policies

    def keep(self, item):
        return any(p.keep(item) for p in self.policies)


def make_policy(names: Sequence[str], dst: BlockManager | None, object_store=None) -> OffloadPolicy:
    ps = []
    for n in names:
        if n == "pass_all":
            ps.append(PassAll())
        elif n == "presence":
            ps.append(PresenceFilter(dst))
        elif n == "presence_lfu":
            ps.append(PresenceAndLFUFilter(dst))
        elif n == "object_presence":
            ps.append(ObjectPresenceFilter(object_store))
        elif n == "object_lock_presence":
            ps.append(ObjectLockPresenceFilter(object_store))
        else:
            raise ValueError(f"unknown offload policy {n!r}")
    return ps[0] if len(ps) == 1 else AllOf(*ps)


# ------------------------------------------------------------------ pipeline
Executor = Callable[[list[OffloadItem]], list[int] | None]


class OffloadPipeline:
    """One tier transition (src -> dst) served by a worker thread."""

    def __init__(self, name: str, dst: BlockManager | None, executor: Executor, policy: OffloadPolicy,
                 cfg: PipelineConfig | None = None, on_registered: Callable[[list[ImmutableBlock]], None] | None = None):
        self.name, self.dst, self.executor, self.policy = name, dst, executor, policy
        self.cfg = cfg or PipelineConfig()
        self.on_registered = on_registered
        self._q: "queue.Queue[OffloadHandle | None]" = queue.Queue()
        self._stop = False
        self.stats = {"enqueued": 0, "offloaded": 0, "filtered": 0, "cancelled": 0, "failed": 0, "batches": 0,
                      "submit_s": 0.0, "complete_s": 0.0}
        self._thread = threading.Thread(target=self._run, name=f"kvbm-offload-{name}", daemon=True)
        self._thread.start()

    def enqueue(self, items: Sequence[OffloadItem], precondition: Callable[[], bool] | None = None) -> OffloadHandle:
        h = OffloadHandle(list(items), precondition)
        self.stats["enqueued"] += len(items)
        self._q.put(h)
        return h

    def _await_precondition(self, h: OffloadHandle) -> bool:
        if h.precondition is None:
            return True
        deadline = time.monotonic() + 60.0
        while not h.precondition():
            if h.cancelled or time.monotonic() > deadline:
                return False
            time.sleep(self.cfg.sweep_ms / 1000.0 / 10)
        return True

    def _run(self) -> None:
        pending: list[tuple[OffloadHandle, list[OffloadItem]]] = []
        last_flush = time.monotonic()
        while not self._stop:
            timeout = self.cfg.flush_ms / 1000.0
            try:
                h = self._q.get(timeout=timeout)
            except queue.Empty:
                h = None
            if h is not None:
                if h.state == OffloadState.CANCELLED:
                    self.stats["cancelled"] += len(h.items)
                else:
                    try:
                        with nvtx_range(f"kvbm.offload.{self.name}.policy"):
                            kept = self.policy.filter(h.items)
                    except Exception as e:  # noqa: BLE001 - a broken policy fails the handle, not the thread
                        h.error = e
                        with h._lock:
                            h._finish(OffloadState.FAILED)
                        self.stats["failed"] += len(h.items)
                        continue
                    h.skipped = [i.seq_hash for i in h.items if i not in kept]
                    self.stats["filtered"] += len(h.items) - len(kept)
                    if not self._await_precondition(h):
                        with h._lock:
                            h._finish(OffloadState.CANCELLED)
                        self.stats["cancelled"] += len(h.items)
                    elif not kept:
                        with h._lock:
                            h._finish(OffloadState.DONE)
                    else:
                        pending.append((h, kept))
            n = sum(len(k) for _, k in pending)
            due = (time.monotonic() - last_flush) * 1000.0 >= self.cfg.flush_ms
            if pending and (n >= self.cfg.min_batch or due or self._q.empty()):
                self._flush(pending)
                pending = []
                last_flush = time.monotonic()

    def _flush(self, pending: list[tuple[OffloadHandle, list[OffloadItem]]]) -> None:
        # split into executor batches of at most max_batch items
        live = []
        for h, items in pending:
            with h._lock:
                if h.cancelled:
                    h._finish(OffloadState.CANCELLED)
                    self.stats["cancelled"] += len(items)
                    continue
                h.state = OffloadState.RUNNING
            live.append((h, items))
        batch: list[tuple[OffloadHandle, OffloadItem]] = [(h, i) for h, items in live for i in items]
        results: dict[int, list] = {id(h): [] for h, _ in live}
        ok = {id(h): True for h, _ in live}
        chunks = [batch[s: s + self.cfg.max_batch] for s in range(0, len(batch), self.cfg.max_batch)]

        def fail(chunk, e):
            for h, _ in chunk:
                ok[id(h)] = False
                h.error = e

        def collect(chunk, reg):
            self.stats["batches"] += 1
            if reg is not None:
                for (h, _), r in zip(chunk, reg):
                    results[id(h)].append(r)

        if hasattr(self.executor, "submit"):
            # launch every batch's copy first, then wait and register in order
            tokens = []
            with nvtx_range(f"kvbm.offload.{self.name}.transfer"):
                t0 = time.perf_counter()
                for chunk in chunks:
                    try:
                        tokens.append((chunk, self.executor.submit([i for _, i in chunk])))
                    except Exception as e:  # noqa: BLE001 - surfaced on the handle
                        fail(chunk, e)
                t1 = time.perf_counter()
                for chunk, tok in tokens:
                    try:
                        collect(chunk, self.executor.complete(tok))
                    except Exception as e:  # noqa: BLE001
                        fail(chunk, e)
                self.stats["submit_s"] += t1 - t0
                self.stats["complete_s"] += time.perf_counter() - t1
        else:
            for chunk in chunks:
                try:
                    with nvtx_range(f"kvbm.offload.{self.name}.transfer"):
                        reg = self.executor([i for _, i in chunk])
                    collect(chunk, reg)
                except Exception as e:  # noqa: BLE001 - surfaced on the handle
                    fail(chunk, e)
        for h, items in live:
            audit("offload_batch", pipeline=self.name, blocks=len(items), ok=ok[id(h)])
            with h._lock:
                if ok[id(h)]:
                    h.registered = [r for r in results[id(h)] if r is not None]
                    self.stats["offloaded"] += len(items)
                    h._finish(OffloadState.DONE)
                else:
                    self.stats["failed"] += len(items)
                    h._finish(OffloadState.FAILED)
            if ok[id(h)] and self.on_registered is not None and h.registered:
                self.on_registered(h.registered)
            # the destination keeps the blocks cached (inactive, matchable);
            # the handle only reports where they went
            h.registered_ids = [(b.sequence_hash, b.block_id) for b in h.registered]
            for b in h.registered:
                b.release()

    def close(self) -> None:
        self._stop = True
        self._thread.join(timeout=5)


class OffloadEngine:
    """Owns the per-transition pipelines and chains G2 registrations into G3."""

    def __init__(self):
        self.pipelines: dict[str, OffloadPipeline] = {}
        self.auto_chain = True

    def add(self, pipeline: OffloadPipeline) -> None:
        self.pipelines[pipeline.name] = pipeline

    def enqueue(self, name: str, items: Sequence[OffloadItem], precondition=None) -> OffloadHandle:
        if name not in self.pipelines:
            raise KeyError(f"no offload pipeline {name!r}")
        return self.pipelines[name].enqueue(items, precondition)

    def enqueue_g1_to_g2_with_precondition(self, items, precondition) -> OffloadHandle:
        return self.enqueue("g1_to_g2", items, precondition)

    def stats(self) -> dict:
        return {k: dict(p.stats) for k, p in self.pipelines.items()}

    def close(self) -> None:
        for p in self.pipelines.values():
            p.close()


class TierExecutor:
    """Allocates destination blocks, transfers into them and registers them.

    ``submit`` allocates and launches the copy without waiting; ``complete``
    waits for it and registers the blocks, so a pipeline can keep several
    batches' copies in flight. Calling the executor does both. With a
    ``journal`` (``engine.tier_journal.TierJournal``, for a persistent G3)
    the destination ids are logged as invalid before the write and as
    committed with their hashes after it.
    """

    def __init__(self, src_handle: int, dst_manager: BlockManager, dst_handle: int, transfer_manager,
                 journal=None):
        self.src_handle, self.dst, self.dst_handle = src_handle, dst_manager, dst_handle
        self.tm, self.journal = transfer_manager, journal

    def submit(self, items: list[OffloadItem]):
        got = self.dst.allocate_blocks_with_evictions(len(items))
        if got is None:
            raise RuntimeError(f"{self.dst.tier.name} pool has no free or evictable blocks")
        blocks, _evicted = got
        dst_ids = [b.block_id for b in blocks]
        if self.journal is not None:
            self.journal.invalidate(dst_ids)
        try:
            note = self.tm.execute_transfer(self.src_handle, [i.src_block_id for i in items], self.dst_handle,
                                            dst_ids)
        except Exception:
            for b in blocks:
                b.release()
            raise
        return items, blocks, note

    def complete(self, token) -> list[ImmutableBlock]:
        items, blocks, note = token
        try:
            note.wait()
        except Exception:
            for b in blocks:
                b.release()
            raise
        if self.journal is not None:
            self.journal.commit([b.block_id for b in blocks], [i.seq_hash for i in items])
        # the registered blocks are cached in the destination's inactive pool
        return list(self.dst.register_mutable(blocks, [i.seq_hash for i in items]))

    def __call__(self, items: list[OffloadItem]) -> list[ImmutableBlock]:
        return self.complete(self.submit(items))


def make_tier_executor(src_handle: int, dst_manager: BlockManager, dst_handle: int, transfer_manager,
                       journal=None) -> TierExecutor:
    """Executor that allocates destination blocks, transfers, and registers them."""
    return TierExecutor(src_handle, dst_manager, dst_handle, transfer_manager, journal)
