"""Worker-side connector: executes the leader's per-step ops on one GPU.

Hooks (called by the serving framework's model runner):

* ``register_kv_caches(tensors)`` / ``register_cross_layers_kv_cache(tensor)``
  / ``register_layout(layout)`` - describe the framework's G1 KV tensors as
  a layout (axis labels from the dimension probe) and build the worker's G2
  (pinned) / G3 (disk) pools;
* ``bind_connector_metadata(raw)`` - the step's ops;
* ``start_load_kv()`` - G3 -> G2 stages and G2 -> G1 onboards on the H2D
  stream (whole blocks, or one transfer per layer with per-layer events in
  intra mode); the H2D stream first waits for earlier offloads so G2 slots
  are never read before they are written. Remote prefills the leader
  dispatched start being watched here;
* ``wait_for_layer_load(layer)`` - intra mode: the compute stream waits on
  that layer's onboard event;
* ``save_kv_layer(layer)`` - on a prefill instance, pushes the blocks of
  remote requests into their decode instance's G1 pool once every
  ``layer_batch`` layers (one fused transfer launch per batch, in the
  compute stream right behind the layer's KV write, NVLink stores into the
  peer's pool);
* ``wait_for_save()`` - G1 -> G2 offloads on the D2H stream behind the
  forward pass, then G2 -> G3 spills; publishes finished pushes (a
  system-scope release store of the request's sequence number into the
  decode instance's host mailbox, behind the last push);
* ``get_finished(finished_req_ids)`` - requests whose onboards completed or
  whose remote prefill's mailbox word landed (``finished_recving``; a word
  that does not land within the timeout reports the request's blocks as
  load errors) and finished requests whose offloads / pushes completed
  (``finished_sending``);
* ``build_connector_worker_meta()`` - the steps whose offload copies this
  worker completed, so the leader registers those G2 blocks only then.

Parity: python/kvbm/vllm/connector/worker.py:74-602 (KvbmConnectorWorker),
crates/kvbm-connector/src/connector/worker/mod.rs:57-275,
crates/kvbm-engine/src/tiering/engine/worker.rs:215-387; the push replaces
the decode side's NIXL pull of the prefill's G2 blocks
(crates/kvbm-engine/src/leader/instance.rs:1394).
"""

from __future__ import annotations

import time

import torch

from ..engine.worker import Worker
from ..physical.layout import KvLayout, LayoutDescriptor
from ..physical.transfer import TransferCapabilities, TransferOptions
from ..utils.config import KvbmConfig
from ..utils.tracing import nvtx_range
from .dim_probe import (KvDim, infer_from_shape, layout_from_cross_layer_tensor, layout_from_layer_tensors)
from .protocol import ConnectorMetadata, PushOp


def blocks_for_bytes(size_gb: float | None, num_blocks: int | None, bytes_per_block: int) -> int:
    if num_blocks:
        return int(num_blocks)
    if size_gb:
        return int(size_gb * (1 << 30)) // bytes_per_block
    return 0


# Instances whose workers live in this process, by (instance, rank): a peer in the same
# process is written through its live pool and mailbox (a CUDA IPC handle cannot be opened by
# the process that exported it).
_LOCAL_SHARDS: dict[tuple[int, int], tuple] = {}


class PeerConnection:
    """A decode instance as a prefill worker writes to it: its G1 pool and mailbox."""

    def __init__(self, info: dict, device: int):
        import os

        from ..parallel.pd import MailboxWriter

        local = _LOCAL_SHARDS.get((info.get("instance"), info.get("rank"))) if info.get("pid") == os.getpid() else None
        if "pool_obj" in info:  # same process (e.g. colocated): the live objects
            self.pool = info["pool_obj"]
            self.mailbox = MailboxWriter(info["mailbox"], local=info["mailbox_obj"])
        elif local is not None:
            self.pool = local[0]
            self.mailbox = MailboxWriter(info["mailbox"], local=local[1])
        else:
            self.pool = KvLayout.from_descriptor(LayoutDescriptor.from_dict(info["pool"]), device=device)
            self.mailbox = MailboxWriter(info["mailbox"])

    def close(self) -> None:
        self.mailbox.close()


_MAPPED_POOLS: dict[str, KvLayout] = {}


def run_remote_pull(op, g2: KvLayout, rank: int) -> int:
    """Copy a remote-search pull into this worker's G2 pool: ``op.src_ids`` of the holder's
    rank-``rank`` G2 pool (a shared-memory file on this node, mapped once and kept) into
    ``op.g2_ids``. Returns the number of blocks copied."""
    from ..engine.remote_search import _map_pool

    pd = op.pools[rank if rank < len(op.pools) else 0]
    path = (pd.get("extra") or {}).get("shm_path") or ""
    src = _MAPPED_POOLS.get(path)
    if src is None:
        src = _map_pool(pd)
        if src is None:
            raise RuntimeError(f"remote pull {op.pull_id}: the holder's G2 pool {path!r} is not on this node")
        _MAPPED_POOLS[path] = src
    g2.scatter_blocks(list(op.g2_ids), src.gather_blocks(list(op.src_ids)))
    return len(op.g2_ids)


class ConnectorWorker:
    def __init__(self, config: KvbmConfig | None = None, rank: int = 0, device: int | None = None,
                 block_size: int = 16, num_kv_heads: int | None = None, head_size: int | None = None):
        self.config = config or KvbmConfig()
        self.rank = rank
        self.device = device if device is not None else (torch.cuda.current_device() if torch.cuda.is_available()
                                                         else 0)
        self.block_size = block_size
        self.num_kv_heads, self.head_size = num_kv_heads, head_size
        self.worker: Worker | None = None
        self.g1: KvLayout | None = None
        self.layer_names: list[str] = []
        self._meta: ConnectorMetadata | None = None
        self._h2d = self._d2h = None
        self._last_offload: torch.cuda.Event | None = None
        self._recv_events: dict[str, torch.cuda.Event] = {}
        self._send_events: dict[str, list[torch.cuda.Event]] = {}
        # requests this worker sent blocks for (offloads, remote-prefill pushes): the only ones whose free
        # the scheduler delays for a send, so the only ones get_finished may report as sent
        self._send_seen: set[str] = set()
        self._layer_events: list[torch.cuda.Event] = []
        self._load_errors: set[int] = set()
        self.transfer_log: list | None = None
        self._pending_finished: set[str] = set()
        self._offload_steps: list[tuple[int, torch.cuda.Event]] = []
        self._pulls_done: list[int] = []  # remote-search pulls copied into G2, reported once
        self._pulls_failed: list[int] = []
        self.objects = None           # engine.object_tier.ObjectTier over this worker's G2 pool (G4 configured)
        self._store_pool = None
        self._stores: list = []       # (step, future) of G2 -> G4 uploads
        self._spill_steps: list[int] = []
        # conditional disaggregation
        self.layer_batch = max(1, int(self.config.transfer.layer_batch))
        self.push_engine = self.config.transfer.push_engine
        self.push_bulk_peer = self.config.transfer.push_bulk_peer
        self.instance_id = 0
        self.directory = None
        self.mailbox = None
        self._peers: dict[int, PeerConnection] = {}
        self._pushes: list[tuple[PushOp, list, torch.Tensor, torch.Tensor]] = []
        self.tp_rank, self.tp_size = 0, 1
        self.landing: KvLayout | None = None   # fp8 landing pool of pushes (wire_dtype="fp8")
        self._recvs: dict[str, tuple] = {}
        self.push_timing = False
        self._push_timers: list[tuple[torch.cuda.Event, torch.cuda.Event, int]] = []
        self.onboard_timing = False   # bracket each step's onboards with CUDA events (take_onboard_timings)
        self._onboard_timers: list[tuple[torch.cuda.Event, torch.cuda.Event, int]] = []

    # --------------------------------------------------------- registration
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor], num_blocks: int | None = None,
                           labels: list[KvDim] | None = None) -> KvLayout:
        self.layer_names = list(kv_caches)
        tensors = [kv_caches[n] for n in self.layer_names]
        t = tensors[0]
        if labels is None:
            if self.num_kv_heads is None or self.head_size is None:
                raise ValueError("num_kv_heads/head_size are needed to label the KV tensors")
            nb = num_blocks or self._guess_blocks(t.shape)
            labels = infer_from_shape(t.shape, nb, self.block_size, self.num_kv_heads, self.head_size)
        nb = t.shape[labels.index(KvDim.BLOCK)]
        heads = t.shape[labels.index(KvDim.HEAD)]
        hd = t.shape[labels.index(KvDim.HEAD_SIZE)]
        # backends may hand out a permuted view of a buffer allocated in another dimension order
        # (a KV stride order): describe the memory in its physical order
        perm = sorted(range(t.dim()), key=lambda i: (-t.stride(i), i))
        if perm != list(range(t.dim())):
            tensors = [x.permute(perm) for x in tensors]
            labels = [labels[i] for i in perm]
        if not all(x.is_contiguous() for x in tensors):
            raise ValueError("KV tensors must be dense (in some dimension order)")
        self.g1 = layout_from_layer_tensors(tensors, labels, nb, self.block_size, heads, hd)
        self._build_worker()
        return self.g1

    def register_cross_layers_kv_cache(self, tensor: torch.Tensor, labels: list[KvDim] | None = None) -> KvLayout:
        if labels is None:
            labels = infer_from_shape(tensor.shape, tensor.shape[0], self.block_size, self.num_kv_heads,
                                      self.head_size, num_layers=tensor.shape[1])
        heads = tensor.shape[labels.index(KvDim.HEAD)]
        hd = tensor.shape[labels.index(KvDim.HEAD_SIZE)]
        self.g1 = layout_from_cross_layer_tensor(tensor, labels, self.block_size, heads, hd)
        self._build_worker()
        return self.g1

    # ------------------------------------------------------------------ G4
    def _fetch(self, op, meta) -> None:
        """Read G4 objects into G2 before the onboard; a missing object makes the blocks it would
        have filled load errors (the framework recomputes them)."""
        if self.objects is None:
            raise RuntimeError("a G4 fetch reached a worker without an object store configured")
        ok = self.objects.get_into(list(op.hashes), list(op.g2_ids))
        bad = {g for g, good in zip(op.g2_ids, ok) if not good}
        if bad:
            for on in meta.onboard:
                if on.req_id == op.req_id:
                    self._load_errors.update(g1 for g2, g1 in zip(on.g2_ids, on.g1_ids) if g2 in bad)

    def _queue_stores(self, meta) -> None:
        """Upload registered G2 blocks to G4 off the forward path; reported with the step."""
        if self.objects is None:
            raise RuntimeError("a G4 store reached a worker without an object store configured")
        import concurrent.futures as cf

        if self._store_pool is None:
            self._store_pool = cf.ThreadPoolExecutor(max_workers=1, thread_name_prefix="kvbm-g4-store")
        ops = [(list(o.hashes), list(o.g2_ids)) for o in meta.store]
        self._stores.append((meta.step, self._store_pool.submit(lambda: [self.objects.put(h, g) for h, g in ops])))

    def publish_g2(self, directory, instance_id: int) -> dict:
        """Publish this worker's G2 pool (a shared-memory file) so another instance on the node can
        pull matched blocks from it (remote search); returns the export."""
        from ..engine.remote_search import pool_export

        d = pool_export(self.worker.g2_layout)
        directory.publish(int(instance_id), d, rank=self.tp_rank if self.tp_size > 1 else self.rank)
        return d

    def register_layout(self, layout: KvLayout) -> KvLayout:
        """Use an already described G1 pool (a serving engine that allocates its KV through the block manager)."""
        self.g1 = layout
        self._build_worker()
        return layout

    def _guess_blocks(self, shape) -> int:
        dims = [d for d in shape[:-1] if d not in (2, self.block_size, self.num_kv_heads)]
        return max(dims) if dims else shape[0]

    def _build_worker(self) -> None:
        c = self.config
        bpb = self.g1.config.bytes_per_block
        g2 = blocks_for_bytes(c.cache.host.cache_size_gb, c.cache.host.num_blocks, bpb)
        g3 = blocks_for_bytes(c.cache.disk.cache_size_gb, c.cache.disk.num_blocks, bpb)
        path = None
        if g3 and c.cache.disk.dir:
            path = f"{c.cache.disk.dir}/kvbm_g3_rank{self.rank}.bin"
        caps = TransferCapabilities(allow_gds=c.transfer.allow_gds, allow_gpu_rdma=c.transfer.allow_gpu_rdma,
                                    cuda_graph_replay=c.transfer.cuda_graph_replay,
                                    startup_benchmark=c.transfer.startup_benchmark)
        self._make_worker(c, g2, g3, path, caps)
        if c.object is not None and g2:
            from ..engine.object_tier import ObjectTier
            from ..object import make_object_store

            self.objects = ObjectTier(make_object_store(c.object), [self.worker.g2_layout], lock=c.object.lock,
                                      rank_base=self.rank)

    def _make_worker(self, c, g2, g3, path, caps) -> None:
        self.worker = Worker(self.rank, self.g1, g2_blocks=g2, g3_blocks=g3, g3_path=path, device=self.device,
                             capabilities=caps, engine=c.transfer.engine, disk_direct=c.cache.disk.use_direct_io,
                             g2_numa_node=c.cache.host.numa_node, g2_hugepages=bool(c.cache.host.hugepages),
                             g2_shared=bool(c.remote_search.enabled))

    def handshake_metadata(self) -> dict:
        """Layout facts the leader needs to size its logical pools."""
        cfg = self.g1.config
        return {"rank": self.rank, "num_layers": cfg.num_layers, "outer_dim": cfg.outer_dim,
                "page_size": cfg.page_size, "inner_dim": cfg.inner_dim, "dtype": cfg.dtype,
                "bytes_per_block": cfg.bytes_per_block, "g1_blocks": cfg.num_blocks,
                "g2_blocks": self.worker.g2_layout.config.num_blocks if self.worker.handles.g2 else 0,
                "g3_blocks": self.worker.g3_layout.config.num_blocks if self.worker.handles.g3 else 0,
                "block_layout": self.g1.block_layout.value, "kind": self.g1.kind}

    # ------------------------------------------- conditional disaggregation
    def enable_disagg(self, instance_id: int, directory, mailbox_slots: int = 0, shared: bool = False,
                      timing: bool = False, tp_rank: int = 0, tp_size: int = 1, wire_dtype: str | None = None) -> None:
        """Join the node's P/D deployment as rank ``tp_rank`` of instance ``instance_id``.

        With ``mailbox_slots`` this worker can receive remote prefills: it
        allocates the host mailbox (a named shared-memory file when
        ``shared``, so prefill workers in other processes map it). Every
        worker publishes its G1 pool (its KV-head shard with tensor
        parallelism), its mailbox and its instance's TP degree in
        ``directory`` and can push (prefill side). ``timing`` brackets each
        push launch with CUDA events (``take_push_timings``).
        """
        from ..parallel.pd import HostMailbox

        self.instance_id, self.directory, self.push_timing = int(instance_id), directory, timing
        self.tp_rank, self.tp_size = int(tp_rank), int(tp_size)
        import os

        info = {"device": self.device, "rank": self.tp_rank, "tp": self.tp_size,
                "heads": self.g1.config.num_heads * self.tp_size, "instance": self.instance_id, "pid": os.getpid()}
        if mailbox_slots:
            name = f"kvbm_mb_{self.instance_id:x}_{self.tp_rank}" if shared else None
            self.mailbox = HostMailbox(mailbox_slots, name=name)
            info["mailbox"] = self.mailbox.descriptor()
            target = self.g1
            if wire_dtype == "fp8":
                from ..physical.layout import LayoutConfig

                c = self.g1.config
                cfg8 = LayoutConfig.for_model(c.num_blocks, c.num_layers, c.num_heads, c.head_dim, c.page_size,
                                              torch.float8_e4m3fn, outer_dim=c.outer_dim)
                self.landing = KvLayout.allocate(cfg8, "fully_contiguous", self.g1.block_layout, fp8_scales=True,
                                                 device=self.device)
                target = self.landing
            info["wire"] = wire_dtype or "native"
            if shared:
                info["pool"] = target.descriptor().to_dict()
                _LOCAL_SHARDS[(self.instance_id, self.tp_rank)] = (target, self.mailbox)
            else:
                info.update(pool_obj=target, mailbox_obj=self.mailbox)
        directory.publish(self.instance_id, info, rank=self.tp_rank)

    def _peer(self, instance: int, rank: int = 0) -> PeerConnection:
        conn = self._peers.get((instance, rank))
        if conn is None:
            conn = self._peers[(instance, rank)] = PeerConnection(self.directory.lookup(instance, rank=rank),
                                                                  self.device)
        return conn

    def _targets(self, peer_tp: int):
        """(decode rank, src head offset, dst head offset, heads, contributor index) for this rank's shard."""
        from ..parallel.tp import ParallelismTemplate, plan_pull, plan_push

        key = (self.tp_size, peer_tp)
        got = getattr(self, "_target_cache", {}).get(key)
        if got is not None:
            return got
        c = self.g1.config
        G = c.num_heads * self.tp_size
        src = ParallelismTemplate(self.tp_size, G, c.num_layers, c.head_dim, c.page_size)
        dst = ParallelismTemplate(peer_tp, G, c.num_layers, c.head_dim, c.page_size)
        pulls = plan_pull(dst, src)
        out = []
        for t in plan_push(src, dst)[self.tp_rank]:
            contrib = [sh.remote_rank for sh in pulls[t.dst_rank].shards].index(self.tp_rank)
            out.append((t.dst_rank, t.src_head_offset, t.dst_head_offset, t.num_heads, contrib))
        self.__dict__.setdefault("_target_cache", {})[key] = out
        return out

    def take_onboard_timings(self) -> tuple[float, int]:
        """(summed device ms of the steps' G2 -> G1 onboards, bytes onboarded) since the last call; waits."""
        ms = nb = 0
        for s, e, b in self._onboard_timers:
            e.synchronize()
            ms += s.elapsed_time(e)
            nb += b
        self._onboard_timers.clear()
        return ms, nb

    def take_push_timings(self) -> tuple[float, int]:
        """(summed device ms of the push launches, bytes pushed) since the last call; waits for them."""
        ms = nb = 0
        for s, e, b in self._push_timers:
            e.synchronize()
            ms += s.elapsed_time(e)
            nb += b
        self._push_timers.clear()
        return ms, nb

    # ----------------------------------------------------------- per step
    def _streams(self):
        if self._h2d is None:
            self._h2d = torch.cuda.Stream(device=self.device, priority=-100)
            self._d2h = torch.cuda.Stream(device=self.device)
        return self._h2d, self._d2h

    def bind_connector_metadata(self, raw: bytes) -> None:
        self._meta = ConnectorMetadata.decode(raw)
        self._pushes = []
        if self.transfer_log is not None:  # which G1 blocks each remote prefill moves (set by tests and tools)
            self.transfer_log += [("push", op.req_id, op.peer, list(op.src_ids), list(op.dst_ids))
                                  for op in self._meta.push]
            self.transfer_log += [("recv", op.req_id, list(op.g1_ids)) for op in self._meta.recv]
        if self._meta.push:
            dev = torch.device("cuda", self.device)
            for op in self._meta.push:
                ids = torch.tensor(op.src_ids + op.dst_ids, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
                n = len(op.src_ids)
                targets = [(self._peer(op.peer, d), so, do, nh, cb) for d, so, do, nh, cb in self._targets(op.peer_tp)]
                self._pushes.append((op, targets, ids[:n], ids[n:]))

    def clear_connector_metadata(self) -> None:
        self._meta = None
        self._pushes = []

    def start_load_kv(self) -> None:
        with nvtx_range("kvbm.connector.start_load_kv"):
            self._start_load_kv()

    def _start_load_kv(self) -> None:
        meta = self._meta
        for op in (meta.pull if meta is not None else ()):
            # host-to-host copy of another instance's G2 blocks; the leader registers them (and only then
            # matches and onboards them) once every worker reported. A failed pull is reported, never
            # raised into the forward pass: the request then prefills what it could not pull.
            try:
                run_remote_pull(op, self.worker.g2_layout, self.tp_rank if self.tp_size > 1 else self.rank)
                self._pulls_done.append(op.pull_id)
            except Exception as e:  # noqa: BLE001
                from ..utils.tracing import audit

                audit("remote_pull_failed", pull=op.pull_id, error=str(e))
                self._pulls_failed.append(op.pull_id)
        now = time.monotonic()
        for op in (meta.recv if meta is not None else ()):
            self._recvs[op.req_id] = (op, now + op.timeout_s)
        if meta is not None and meta.store:
            self._queue_stores(meta)
        if meta is None or not (meta.onboard or meta.stage or meta.fetch):
            self._layer_events = []
            return
        h2d, _ = self._streams()
        if self._last_offload is not None:
            h2d.wait_event(self._last_offload)
        intra = self.config.onboard.mode == "intra"
        w = self.worker
        for op in meta.stage:  # G3 -> G2 ahead of the onboards that read them
            w.tm.execute_transfer(w.handles.g3, op.g3_ids, w.handles.g2, op.g2_ids,
                                  TransferOptions(stream=h2d, engine=w.engine)).wait()
        for op in meta.fetch:  # G4 -> G2 ahead of the onboards that read them
            self._fetch(op, meta)
        self._layer_events = []
        if not meta.onboard:
            return
        t0 = None
        if self.onboard_timing:
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(h2d)
        if intra:
            g2 = [i for op in meta.onboard for i in op.g2_ids]
            g1 = [i for op in meta.onboard for i in op.g1_ids]
            for l in range(self.g1.config.num_layers):
                w.tm.execute_transfer(w.handles.g2, g2, w.handles.g1, g1,
                                      TransferOptions(layer_range=(l, l + 1), stream=h2d, engine=w.engine))
                ev = torch.cuda.Event()
                ev.record(h2d)
                self._layer_events.append(ev)
            for op in meta.onboard:
                self._recv_events[op.req_id] = self._layer_events[-1]
        else:
            for op in meta.onboard:
                w.tm.execute_transfer(w.handles.g2, op.g2_ids, w.handles.g1, op.g1_ids,
                                      TransferOptions(stream=h2d, engine=w.engine))
                ev = torch.cuda.Event()
                ev.record(h2d)
                self._recv_events[op.req_id] = ev
            # inter mode: the whole onboard completes before the forward pass
            torch.cuda.current_stream(self.device).wait_stream(h2d)
        if t0 is not None:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record(h2d)
            nblk = sum(len(op.g1_ids) for op in meta.onboard)
            self._onboard_timers.append((t0, t1, nblk * self.g1.config.bytes_per_block))

    def wait_for_layer_load(self, layer: int | str) -> None:
        if isinstance(layer, str):
            layer = self.layer_names.index(layer)
        if layer < len(self._layer_events):
            torch.cuda.current_stream(self.device).wait_event(self._layer_events[layer])

    def save_kv_layer(self, layer: int | str, requests=None) -> None:
        """Push the remote requests' layers once a batch of ``layer_batch`` layers is written.

        ``requests`` limits the pushes to those requests (a runner that runs
        its requests' forward passes one at a time calls this per request);
        None pushes every remote request of the step.
        """
        if not self._pushes:
            return
        if isinstance(layer, str):
            layer = self.layer_names.index(layer)
        nl = self.g1.config.num_layers
        lb = self.layer_batch
        if (layer + 1) % lb and layer != nl - 1:
            return
        first = layer - (layer % lb)
        st = torch.cuda.current_stream(self.device)
        from ..ops import kv_ops

        with nvtx_range(f"kvbm.connector.push.layers{first}-{layer}"):
            self._push_batch(first, layer, st, requests, kv_ops)

    def _push_batch(self, first: int, layer: int, st, requests, kv_ops) -> None:
        for op, targets, src, dst in self._pushes:
            if requests is not None and op.req_id not in requests:
                continue
            for conn, so, do, nh, _ in targets:
                if self.push_timing:
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record(st)
                kv_ops.kv_transfer(self.g1, src, conn.pool, dst, layer_begin=first, num_layers=layer + 1 - first,
                                   src_head_offset=so, dst_head_offset=do, num_heads=nh, engine=self.push_engine,
                                   stream=st, bulk=True if self.push_bulk_peer else None)
                if self.push_timing:
                    e.record(st)
                    c = self.g1.config
                    self._push_timers.append((s, e, len(op.src_ids) * (layer + 1 - first) * c.outer_dim
                                              * c.bytes_per_chunk * nh // c.num_heads))

    def wait_for_save(self) -> None:
        with nvtx_range("kvbm.connector.wait_for_save"):
            self._wait_for_save()

    def _wait_for_save(self) -> None:
        meta = self._meta
        if meta is None:
            return
        from ..ops import kv_ops

        st = torch.cuda.current_stream(self.device)
        for op, targets, _, _ in self._pushes:
            if op.final:
                # behind the request's last push in stream order: the decode side may read its blocks
                for conn, _, _, _, cb in targets:
                    kv_ops.signal_flag(conn.mailbox.flag_ptr(op.slot, cb), op.seq, stream=st)
                ev = torch.cuda.Event()
                ev.record(st)
                self._send_events.setdefault(op.req_id, []).append(ev)
                self._send_seen.add(op.req_id)
        if not (meta.offload or meta.spill):
            return
        _, d2h = self._streams()
        d2h.wait_stream(st)
        w = self.worker
        for op in meta.offload:
            w.tm.execute_transfer(w.handles.g1, op.g1_ids, w.handles.g2, op.g2_ids,
                                  TransferOptions(stream=d2h, engine=w.engine))
            ev = torch.cuda.Event()
            ev.record(d2h)
            self._send_events.setdefault(op.req_id, []).append(ev)
            self._send_seen.add(op.req_id)
            self._last_offload = ev
        if meta.offload:
            self._offload_steps.append((meta.step, self._last_offload))
        for op in meta.spill:  # G2 -> G3 (the sources were registered after their offload landed)
            w.tm.execute_transfer(w.handles.g2, op.g2_ids, w.handles.g3, op.g3_ids,
                                  TransferOptions(engine=w.engine)).wait()
        if meta.spill:
            self._spill_steps.append(meta.step)

    def get_finished(self, finished_req_ids: set[str] | None = None) -> tuple[set[str], set[str]]:
        recving = {r for r, ev in self._recv_events.items() if ev.query()}
        for r in recving:
            del self._recv_events[r]
        if self._recvs:
            now = time.monotonic()
            for r, (op, deadline) in list(self._recvs.items()):
                if r in self._recv_events:
                    continue  # its local onboard part is still running
                if self.mailbox is not None and self.mailbox.landed(op.slot, op.seq, op.contributors):
                    del self._recvs[r]
                    if self.landing is not None:
                        # fp8 on the wire: dequantise into G1, report once that copy is done
                        from ..ops import kv_ops

                        h2d, _ = self._streams()
                        kv_ops.kv_transfer(self.landing, op.g1_ids, self.g1, op.g1_ids, engine="tile", stream=h2d)
                        ev = torch.cuda.Event()
                        ev.record(h2d)
                        self._recv_events[r] = ev
                    else:
                        recving.add(r)
                elif now > deadline:
                    # the prefill never published: report the blocks so the framework recomputes them
                    self._load_errors.update(op.g1_ids)
                    recving.add(r)
                    del self._recvs[r]
        recving -= set(self._recvs)
        # a finished request is reported sent once its copies are done, and only if it sent any: a
        # request the scheduler freed at once must not come back (vLLM no longer knows it)
        self._pending_finished |= set(finished_req_ids or ()) & self._send_seen
        sending = set()
        for r in list(self._pending_finished):
            evs = self._send_events.get(r)
            if not evs or all(ev.query() for ev in evs):
                sending.add(r)
                self._pending_finished.discard(r)
                self._send_events.pop(r, None)
                self._send_seen.discard(r)
        return sending, recving

    def build_connector_worker_meta(self) -> dict | None:
        """Steps whose G1 -> G2 copies this worker finished (the leader registers their G2 blocks then)."""
        done = {}
        while self._offload_steps and self._offload_steps[0][1].query():
            step, _ = self._offload_steps.pop(0)
            done[step] = 1
        spilled = {s: 1 for s in self._spill_steps}
        self._spill_steps = []
        out = {}
        if done:
            out["offloaded"] = done
        if spilled:
            out["spilled"] = spilled
        if self._pulls_done:
            out["pulled"] = {p: 1 for p in self._pulls_done}
            self._pulls_done = []
        if self._pulls_failed:
            out["pull_failed"] = {p: 1 for p in self._pulls_failed}
            self._pulls_failed = []
        stored = {}
        while self._stores and self._stores[0][1].done():
            step, fut = self._stores.pop(0)
            fut.result()  # an upload error surfaces here
            stored[step] = 1
        if stored:
            out["stored"] = stored
        return out or None

    def get_block_ids_with_load_errors(self) -> set[int]:
        out, self._load_errors = self._load_errors, set()
        return out

    def handle_preemptions(self, preempted_req_ids) -> None:
        """Fence: wait for in-flight offloads of preempted requests before their G1 blocks are reused."""
        for r in preempted_req_ids or ():
            for ev in self._send_events.pop(r, []):
                ev.synchronize()

    def shutdown(self) -> None:
        # leave the node's directory first: a pool entry outliving this process would name IPC
        # handles nobody can open any more
        withdraw = getattr(self.directory, "withdraw", None)
        if withdraw is not None:
            try:
                withdraw(self.instance_id, rank=self.tp_rank)
            except OSError:
                pass
        for c in self._peers.values():
            c.close()
        self._peers.clear()
        if self.mailbox is not None:
            _LOCAL_SHARDS.pop((self.instance_id, self.tp_rank), None)
            self.mailbox.close()
            self.mailbox = None
        if self._store_pool is not None:
            self._store_pool.shutdown(wait=True)
        if self.worker is not None:
            self.worker.close()
