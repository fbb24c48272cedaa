"""Replicated-data (MLA) parallelism: one rank owns the lower tiers and
replicates loaded G1 blocks to every other rank.

With MLA-style models every TP rank holds the *same* KV, so only rank 0
keeps G2/G3; after rank 0 onboards blocks into its G1 they are broadcast to
the other ranks' G1.

* :class:`P2PFanoutCollectives` - the product path: rank 0 maps every
  peer's G1 pool through CUDA IPC and writes the blocks straight into each
  peer's paged slots with the fused transfer kernel (one launch per peer,
  NVLink stores), then publishes a per-peer completion flag; peers make
  their compute stream wait on the flag with a bounded-spin kernel.
* :class:`NcclCollectives` - the baseline: gather the blocks into a
  contiguous staging buffer, ``torch.distributed.broadcast`` it over NCCL,
  scatter on every rank.
* :class:`StubCollectives` - single rank, nothing to do.

Parity: crates/kvbm-engine/src/collectives/{mod.rs:75-113 (CollectiveOps:
broadcast(src, dst, src_ids, dst_ids, layer_range), rank, world_size),
nccl.rs:156-482 (NcclCollectives, one ncclBcast per region inside a group),
stub.rs}, worker/physical/replicated.rs:50-150 (ReplicatedDataWorker).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kv_ops
from ..physical.layout import KvLayout, LayoutConfig, LayoutDescriptor
from ..physical.memory import DeviceBuffer, PeerBuffer

WAIT_NS = 30_000_000_000


class CollectiveOps:
    rank: int = 0
    world_size: int = 1

    def broadcast(self, src_ids: list[int], dst_ids: list[int], layer_range: tuple[int, int] | None = None,
                  stream: torch.cuda.Stream | None = None) -> None:
        raise NotImplementedError


class StubCollectives(CollectiveOps):
    def broadcast(self, src_ids, dst_ids, layer_range=None, stream=None) -> None:
        if dist.is_initialized() and dist.get_world_size() > 1:
            raise RuntimeError("StubCollectives used with more than one rank")


class NcclCollectives(CollectiveOps):
    """Baseline: gather -> NCCL broadcast -> scatter."""

    def __init__(self, g1: KvLayout, group=None, max_blocks: int = 64):
        self.g1, self.group = g1, group
        self.rank = dist.get_rank(group)
        self.world_size = dist.get_world_size(group)
        cfg = g1.config
        self.max_blocks = max_blocks
        self.staging = torch.empty(max_blocks * cfg.bytes_per_block, dtype=torch.uint8, device=g1.device)
        self.stage_layout = KvLayout.over_tensor(LayoutConfig(**{**cfg.__dict__, "num_blocks": max_blocks}),
                                                 self.staging, "fully_contiguous", g1.block_layout)

    def broadcast(self, src_ids, dst_ids, layer_range=None, stream=None) -> None:
        lb, le = layer_range or (0, self.g1.config.num_layers)
        for s in range(0, len(dst_ids), self.max_blocks):
            d = dst_ids[s: s + self.max_blocks]
            seq = list(range(len(d)))
            if self.rank == 0:
                kv_ops.kv_transfer(self.g1, src_ids[s: s + self.max_blocks], self.stage_layout, seq,
                                   layer_begin=lb, num_layers=le - lb)
            dist.broadcast(self.staging[: len(d) * self.g1.config.bytes_per_block], src=dist.get_global_rank(
                self.group, 0) if self.group is not None else 0, group=self.group)
            if self.rank != 0:
                kv_ops.kv_transfer(self.stage_layout, seq, self.g1, d, layer_begin=lb, num_layers=le - lb)


class P2PFanoutCollectives(CollectiveOps):
    """Product path: rank 0 stores into every peer's G1 over NVLink."""

    def __init__(self, g1: KvLayout, group=None, engine: str = "tma"):
        self.g1, self.group, self.engine = g1, group, engine
        self.rank = dist.get_rank(group)
        self.world_size = dist.get_world_size(group)
        self.flags = DeviceBuffer(4096, zero=True)  # [0] completion sequence, [8] status
        self.seq = 0
        mine = (g1.descriptor().to_dict(), self.flags.ipc_handle())
        everyone = [None] * self.world_size
        dist.all_gather_object(everyone, mine, group=self.group)
        self.peers: list[tuple[KvLayout, PeerBuffer]] = []
        if self.rank == 0:
            for r in range(1, self.world_size):
                desc, fh = everyone[r]
                self.peers.append((KvLayout.from_descriptor(LayoutDescriptor.from_dict(desc)),
                                   PeerBuffer(fh, 4096)))

    def broadcast(self, src_ids, dst_ids, layer_range=None, stream=None) -> None:
        """Asynchronous on ``stream``: peers' streams wait on the flag, not the host."""
        self.seq += 1
        lb, le = layer_range or (0, self.g1.config.num_layers)
        st = stream or torch.cuda.current_stream()
        if self.rank == 0:
            dev = self.g1.device
            sid = torch.tensor(src_ids, dtype=torch.int32, device=dev)
            did = torch.tensor(dst_ids, dtype=torch.int32, device=dev)
            for peer, flag in self.peers:
                kv_ops.kv_transfer(self.g1, sid, peer, did, layer_begin=lb, num_layers=le - lb,
                                   engine=self.engine, stream=st)
                kv_ops.signal_flag(flag.ptr, self.seq, stream=st)
        else:
            kv_ops.wait_flag(self.flags.ptr, self.seq, WAIT_NS, self.flags.ptr + 8, stream=st)

    def check(self) -> None:
        st = int(self.flags.tensor(torch.int32)[2].item())
        if st != 0:
            raise TimeoutError("replicated-data broadcast wait timed out")


class ReplicatedDataWorker:
    """Rank 0 onboards from its G2/G3, then replicates to all ranks."""

    def __init__(self, worker, collectives: CollectiveOps):
        self.worker, self.coll = worker, collectives

    def onboard(self, g2_ids: list[int] | None, g1_ids: list[int], stream=None) -> None:
        from ..logical.manager import Tier

        if self.coll.rank == 0 and g2_ids:
            self.worker.execute_local_transfer(Tier.G2, g2_ids, Tier.G1, g1_ids).wait()
        self.coll.broadcast(g1_ids, g1_ids, stream=stream)
