"""Worker-side connector: executes the leader's per-step ops on one GPU.

Hooks (called by the serving framework's model runner):

* ``register_kv_caches(tensors)`` / ``register_cross_layers_kv_cache(tensor)``
  - describe the framework's G1 KV tensors as a layout (axis labels from the
  dimension probe) and build the worker's G2 (pinned) / G3 (disk) pools;
* ``bind_connector_metadata(raw)`` - the step's onboard/offload ops;
* ``start_load_kv()`` - G2 -> G1 onboards on the H2D stream (whole blocks,
  or one transfer per layer with per-layer events in intra mode); the H2D
  stream first waits for earlier offloads so G2 slots are never read before
  they are written;
* ``wait_for_layer_load(layer)`` - intra mode: the compute stream waits on
  that layer's onboard event;
* ``save_kv_layer(layer)`` - records the layer's compute event;
* ``wait_for_save()`` - G1 -> G2 offloads on the D2H stream behind the
  forward pass;
* ``get_finished(finished_req_ids)`` - requests whose onboards completed
  (``finished_recving``) and finished requests whose offloads completed
  (``finished_sending``).

Parity: python/kvbm/vllm/connector/worker.py:74-602 (KvbmConnectorWorker),
crates/kvbm-connector/src/connector/worker/mod.rs:57-275,
crates/kvbm-engine/src/tiering/engine/worker.rs:215-387.
"""

from __future__ import annotations

import torch

from ..engine.worker import Worker
from ..physical.layout import KvLayout
from ..physical.transfer import TransferCapabilities, TransferOptions
from ..utils.config import KvbmConfig
from .dim_probe import (KvDim, infer_from_shape, layout_from_cross_layer_tensor, layout_from_layer_tensors)
from .protocol import ConnectorMetadata


def blocks_for_bytes(size_gb: float | None, num_blocks: int | None, bytes_per_block: int) -> int:
    if num_blocks:
        return int(num_blocks)
    if size_gb:
        return int(size_gb * (1 << 30)) // bytes_per_block
    return 0


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
        self._send_events: dict[str, torch.cuda.Event] = {}
        self._layer_events: list[torch.cuda.Event] = []
        self._load_errors: set[int] = set()
        self._pending_finished: set[str] = set()

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
        self.worker = Worker(self.rank, self.g1, g2_blocks=g2, g3_blocks=g3, g3_path=path, device=self.device,
                             capabilities=caps, engine=c.transfer.engine, disk_direct=c.cache.disk.use_direct_io,
                             g2_numa_node=c.cache.host.numa_node, g2_hugepages=bool(c.cache.host.hugepages))

    def handshake_metadata(self) -> dict:
        """Layout facts the leader needs to size its logical pools."""
        cfg = self.g1.config
        return {"rank": self.rank, "num_layers": cfg.num_layers, "outer_dim": cfg.outer_dim,
                "page_size": cfg.page_size, "inner_dim": cfg.inner_dim, "dtype": cfg.dtype,
                "bytes_per_block": cfg.bytes_per_block, "g1_blocks": cfg.num_blocks,
                "g2_blocks": self.worker.g2_layout.config.num_blocks if self.worker.handles.g2 else 0,
                "g3_blocks": self.worker.g3_layout.config.num_blocks if self.worker.handles.g3 else 0,
                "block_layout": self.g1.block_layout.value, "kind": self.g1.kind}

    # ----------------------------------------------------------- per step
    def _streams(self):
        if self._h2d is None:
            self._h2d = torch.cuda.Stream(device=self.device, priority=-100)
            self._d2h = torch.cuda.Stream(device=self.device)
        return self._h2d, self._d2h

    def bind_connector_metadata(self, raw: bytes) -> None:
        self._meta = ConnectorMetadata.decode(raw)

    def clear_connector_metadata(self) -> None:
        self._meta = None

    def start_load_kv(self) -> None:
        if self._meta is None or not self._meta.onboard:
            self._layer_events = []
            return
        h2d, _ = self._streams()
        if self._last_offload is not None:
            h2d.wait_event(self._last_offload)
        intra = self.config.onboard.mode == "intra"
        w = self.worker
        self._layer_events = []
        if intra:
            g2 = [i for op in self._meta.onboard for i in op.g2_ids]
            g1 = [i for op in self._meta.onboard for i in op.g1_ids]
            for l in range(self.g1.config.num_layers):
                w.tm.execute_transfer(w.handles.g2, g2, w.handles.g1, g1,
                                      TransferOptions(layer_range=(l, l + 1), stream=h2d, engine=w.engine))
                ev = torch.cuda.Event()
                ev.record(h2d)
                self._layer_events.append(ev)
            for op in self._meta.onboard:
                self._recv_events[op.req_id] = self._layer_events[-1]
        else:
            for op in self._meta.onboard:
                w.tm.execute_transfer(w.handles.g2, op.g2_ids, w.handles.g1, op.g1_ids,
                                      TransferOptions(stream=h2d, engine=w.engine))
                ev = torch.cuda.Event()
                ev.record(h2d)
                self._recv_events[op.req_id] = ev
            # inter mode: the whole onboard completes before the forward pass
            torch.cuda.current_stream(self.device).wait_stream(h2d)

    def wait_for_layer_load(self, layer: int | str) -> None:
        if isinstance(layer, str):
            layer = self.layer_names.index(layer)
        if layer < len(self._layer_events):
            torch.cuda.current_stream(self.device).wait_event(self._layer_events[layer])

    def save_kv_layer(self, layer: int | str) -> None:
        # whole-pass offload (wait_for_save) needs no per-layer event; intra-pass
        # offload would record one here
        return None

    def wait_for_save(self) -> None:
        if self._meta is None or not self._meta.offload:
            return
        _, d2h = self._streams()
        d2h.wait_stream(torch.cuda.current_stream(self.device))
        w = self.worker
        for op in self._meta.offload:
            w.tm.execute_transfer(w.handles.g1, op.g1_ids, w.handles.g2, op.g2_ids,
                                  TransferOptions(stream=d2h, engine=w.engine))
            ev = torch.cuda.Event()
            ev.record(d2h)
            self._send_events[op.req_id] = ev
            self._last_offload = ev

    def get_finished(self, finished_req_ids: set[str] | None = None) -> tuple[set[str], set[str]]:
        recving = {r for r, ev in self._recv_events.items() if ev.query()}
        for r in recving:
            del self._recv_events[r]
        self._pending_finished |= set(finished_req_ids or ())
        sending = set()
        for r in list(self._pending_finished):
            ev = self._send_events.get(r)
            if ev is None or ev.query():
                sending.add(r)
                self._pending_finished.discard(r)
                self._send_events.pop(r, None)
        return sending, recving

    def get_block_ids_with_load_errors(self) -> set[int]:
        out, self._load_errors = self._load_errors, set()
        return out

    def handle_preemptions(self, preempted_req_ids) -> None:
        """Fence: wait for in-flight offloads of preempted requests before their G1 blocks are reused."""
        for r in preempted_req_ids or ():
            ev = self._send_events.pop(r, None)
            if ev is not None:
                ev.synchronize()

    def shutdown(self) -> None:
        if self.worker is not None:
            self.worker.close()
