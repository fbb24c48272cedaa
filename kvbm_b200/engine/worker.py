"""Workers: the processes that own GPU memory and execute transfers.

A :class:`Worker` (one per GPU / TP rank) owns a ``TransferManager`` with
the G1 layout (the serving framework's KV tensors), a pinned G2 pool, an
optional G3 disk pool and the staging bounce buffer. The leader only decides
*which* blocks move; workers move bytes.

Layer-wise onboarding (``OnboardMode.intra``): one G2 -> G1 transfer per
layer on the H2D stream, each followed by an event; the forward pass makes
its compute stream wait on layer ``l``'s event right before layer ``l``'s
attention, so loading overlaps the earlier layers' compute. Layer-wise
offload records a compute event after each layer's KV is written and runs
the layer's G1 -> G2 copy on the D2H stream behind it.

Parity: crates/kvbm-engine/src/worker/{mod.rs:38-209 (WorkerTransfers,
Worker), physical.rs:189-440 (resolve_layout, create_bounce_buffer,
export/import_metadata, execute_local_layerwise_onboard)},
crates/kvbm-engine/src/tiering/engine/worker.rs:123-387 (per-layer onboard
and compute events, offload-complete event).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from ..logical.manager import Tier
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig
from ..physical.transfer import (DiskLayout, SerializedLayouts, TransferCapabilities,
                                 TransferCompleteNotification, TransferManager, TransferOptions)


@dataclass
class WorkerLayouts:
    g1: int
    g2: int | None = None
    g3: int | None = None
    bounce: int | None = None


class Worker:
    def __init__(self, rank: int, g1: KvLayout, g2_blocks: int = 0, g3_blocks: int = 0, g3_path: str | None = None,
                 device: int | None = None, capabilities: TransferCapabilities | None = None,
                 engine: str = "auto", bounce_blocks: int = 64, disk_direct: bool = True,
                 g2_numa_node: int | str | None = None, g2_hugepages: bool = False, g2_shared: bool = False):
        self.rank = rank
        self.device = device if device is not None else (g1.device if g1.device is not None else 0)
        self.tm = TransferManager(worker_id=rank, device=self.device, capabilities=capabilities)
        self.engine = engine
        self.g1_layout = g1
        self.handles = WorkerLayouts(g1=self.tm.register_layout(g1))
        cfg = g1.config
        fc = KvBlockLayout.OPERATIONAL_NHD if g1.block_layout == KvBlockLayout.UNIVERSAL else g1.block_layout
        if g2_blocks:
            g2cfg = LayoutConfig(**{**cfg.__dict__, "num_blocks": g2_blocks})
            # g2_shared: a named shared-memory file other instances on the node can map (remote search)
            self.g2_layout = KvLayout.allocate(g2cfg, "fully_contiguous", fc,
                                               location="shared" if g2_shared else "pinned", device=self.device,
                                               numa_node=None if g2_shared else g2_numa_node,
                                               hugepages=False if g2_shared else g2_hugepages)
            self.handles.g2 = self.tm.register_layout(self.g2_layout)
        if g3_blocks:
            g3cfg = LayoutConfig(**{**cfg.__dict__, "num_blocks": g3_blocks})
            path = g3_path or f"/tmp/kvbm_g3_{rank}_{id(self)}.bin"
            self.g3_layout = DiskLayout(g3cfg, path, direct=disk_direct, block_layout=fc)
            self.handles.g3 = self.tm.register_layout(self.g3_layout)
            bcfg = LayoutConfig(**{**cfg.__dict__, "num_blocks": bounce_blocks})
            self.bounce = KvLayout.allocate(bcfg, "fully_contiguous", fc, location="pinned")
            self.tm.set_bounce(self.bounce)
        self._h2d = None
        self._d2h = None
        self.onboard_events: list[torch.cuda.Event] = []
        self.compute_events: list[torch.cuda.Event] = []
        self._lock = threading.Lock()

    # ------------------------------------------------------------- lookup
    def handle(self, tier: Tier) -> int:
        h = {Tier.G1: self.handles.g1, Tier.G2: self.handles.g2, Tier.G3: self.handles.g3}.get(Tier(tier))
        if h is None:
            raise ValueError(f"worker {self.rank} has no {Tier(tier).name} layout")
        return h

    def export_metadata(self) -> SerializedLayouts:
        return self.tm.export_metadata()

    def import_metadata(self, meta: SerializedLayouts) -> dict[int, int]:
        return self.tm.import_metadata(meta)

    # ---------------------------------------------------------- transfers
    def execute_local_transfer(self, src_tier: Tier, src_ids, dst_tier: Tier, dst_ids,
                               layer_range: tuple[int, int] | None = None,
                               head_range: tuple[int, int, int] | None = None) -> TransferCompleteNotification:
        return self.tm.execute_transfer(self.handle(src_tier), src_ids, self.handle(dst_tier), dst_ids,
                                        TransferOptions(layer_range=layer_range, head_range=head_range,
                                                        engine=self.engine))

    def execute_remote_transfer(self, src_tier: Tier, src_ids, remote_handle: int, dst_ids,
                                layer_range=None, head_range=None) -> TransferCompleteNotification:
        """Push local blocks into a peer's mapped G1 pool (P2P over NVLink)."""
        return self.tm.execute_transfer(self.handle(src_tier), src_ids, remote_handle, dst_ids,
                                        TransferOptions(layer_range=layer_range, head_range=head_range,
                                                        engine=self.engine if self.engine != "auto" else "tma"))

    # ------------------------------------------------- layer-wise onboard
    def _streams(self):
        if self._h2d is None:
            self._h2d = torch.cuda.Stream(device=self.device, priority=-100)
            self._d2h = torch.cuda.Stream(device=self.device)
        return self._h2d, self._d2h

    def start_layerwise_onboard(self, g2_ids, g1_ids) -> None:
        """Enqueue one G2 -> G1 transfer per layer, each followed by its event."""
        h2d, _ = self._streams()
        L = self.g1_layout.config.num_layers
        self.onboard_events = []
        for l in range(L):
            self.tm.execute_transfer(self.handles.g2, g2_ids, self.handles.g1, g1_ids,
                                     TransferOptions(layer_range=(l, l + 1), stream=h2d, engine=self.engine))
            ev = torch.cuda.Event()
            ev.record(h2d)
            self.onboard_events.append(ev)

    def wait_for_layer_load(self, layer: int, stream: torch.cuda.Stream | None = None) -> None:
        if layer < len(self.onboard_events):
            (stream or torch.cuda.current_stream()).wait_event(self.onboard_events[layer])

    def save_kv_layer(self, layer: int, stream: torch.cuda.Stream | None = None) -> torch.cuda.Event:
        ev = torch.cuda.Event()
        ev.record(stream or torch.cuda.current_stream())
        while len(self.compute_events) <= layer:
            self.compute_events.append(None)
        self.compute_events[layer] = ev
        return ev

    def offload_layer(self, layer: int, g1_ids, g2_ids) -> TransferCompleteNotification:
        """G1 -> G2 for one layer, behind that layer's compute event (intra-pass offload)."""
        _, d2h = self._streams()
        ev = self.compute_events[layer] if layer < len(self.compute_events) else None
        if ev is not None:
            d2h.wait_event(ev)
        self.tm.execute_transfer(self.handles.g1, g1_ids, self.handles.g2, g2_ids,
                                 TransferOptions(layer_range=(layer, layer + 1), stream=d2h, engine=self.engine))
        done = torch.cuda.Event()
        done.record(d2h)
        return TransferCompleteNotification(event=done)

    def close(self) -> None:
        self.tm.close()
