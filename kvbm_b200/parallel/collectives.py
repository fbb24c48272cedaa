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
* :class:`NvlsFanoutCollectives` - the one-to-many path through NVSwitch
  multicast: every rank's G1 pool lives in one symmetric-memory allocation
  bound to an NVLink multicast object, and rank 0 writes each chunk once with
  ``multimem.st`` (the switch replicates it to every member), then bumps the
  group's completion counter through the same multicast address. Rank 0
  sends the bytes over NVLink once instead of ``world_size - 1`` times.
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
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig, LayoutDescriptor
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


class NvlsUnavailable(RuntimeError):
    """The GPUs or the driver offer no NVLink multicast object for this group."""


class NvlsFanoutCollectives(CollectiveOps):
    """Rank 0 fans blocks out to every rank with one multicast store per 16 bytes."""

    FLAG_BYTES = 4096

    @staticmethod
    def allocate_pool(config: LayoutConfig, group=None, kind: str = "fully_contiguous",
                      block_layout: KvBlockLayout = KvBlockLayout.OPERATIONAL_NHD):
        """Collective: allocate this rank's replicated G1 pool (plus a completion-counter page) in
        symmetric memory and bind it to the group's multicast object. Returns ``(layout, handle,
        flag_offset)``; ``handle.multicast_ptr`` is 0 when the platform has no multicast."""
        import torch.distributed._symmetric_memory as symm

        if block_layout == KvBlockLayout.UNIVERSAL:
            raise ValueError("the multicast fan-out copies contiguous (block, layer, K/V) chunks")
        *_, data = KvLayout._strides(config, kind, block_layout, True)
        flag_off = (data + 4095) // 4096 * 4096
        dev = torch.device("cuda", torch.cuda.current_device())
        t = symm.empty(flag_off + NvlsFanoutCollectives.FLAG_BYTES, dtype=torch.uint8, device=dev)
        t.zero_()
        handle = symm.rendezvous(t, group if group is not None else dist.group.WORLD)
        layout = KvLayout.over_tensor(config, t, kind, block_layout)
        layout._symm = (t, handle)
        torch.cuda.synchronize()
        dist.barrier(group=group)
        return layout, handle, flag_off

    def __init__(self, g1: KvLayout, handle, flag_offset: int, group=None, max_ctas: int = 0,
                 wait_ns: int = WAIT_NS):
        self.g1, self.group = g1, group
        self.rank = dist.get_rank(group)
        self.world_size = dist.get_world_size(group)
        self.mc = int(getattr(handle, "multicast_ptr", 0) or 0)
        if not self.mc:
            raise NvlsUnavailable("no NVLink multicast object for this group")
        self.handle = handle
        self.flag_ptr = g1.base_ptr + flag_offset
        self.flag_mc = self.mc + flag_offset
        self.max_ctas, self.wait_ns = max_ctas, wait_ns
        self.cta_done = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", g1.device))
        self.status = torch.zeros(2, dtype=torch.int32, device=self.cta_done.device)
        self.seq = 0

    def broadcast(self, src_ids, dst_ids, layer_range=None, stream=None) -> None:
        """Asynchronous on ``stream``: every rank's stream (rank 0's included) waits for the
        group counter to reach this call's sequence number."""
        import ctypes

        from ..ops import _lib

        self.seq += 1
        cfg = self.g1.config
        lb, le = layer_range or (0, cfg.num_layers)
        st = stream or torch.cuda.current_stream()
        if len(src_ids) != len(dst_ids):
            raise ValueError("src_ids and dst_ids differ in length")
        nb = cfg.num_blocks
        if any(not 0 <= int(i) < nb for i in list(src_ids) + list(dst_ids)):
            raise IndexError(f"block id outside [0, {nb})")
        if self.rank == 0 and len(dst_ids):
            dev = self.cta_done.device
            sid = torch.as_tensor(src_ids, dtype=torch.int32).to(dev, non_blocking=True)
            did = torch.as_tensor(dst_ids, dtype=torch.int32).to(dev, non_blocking=True)
            n = le - lb
            src_base = (ctypes.c_uint64 * n)(*[self.g1.layer_base(l) for l in range(lb, le)])
            dst_off = (ctypes.c_uint64 * n)(*[self.g1.layer_offsets[l] for l in range(lb, le)])
            _lib.call("kvbm_kv_multicast", src_base, dst_off, n, self.mc, self.g1.block_stride,
                      self.g1.outer_stride, cfg.bytes_per_chunk, cfg.outer_dim, sid.data_ptr(), did.data_ptr(),
                      len(dst_ids), nb, self.flag_mc, self.cta_done.data_ptr(), self.status.data_ptr() + 4,
                      self.max_ctas, kv_ops._stream(st))
            self._keep = (sid, did)
        elif self.rank == 0:
            # nothing to copy: still advance every member's counter so the sequence stays aligned
            kv_ops.signal_flag_multicast(self.flag_mc, stream=st)
        kv_ops.wait_flag(self.flag_ptr, self.seq, self.wait_ns, self.status.data_ptr(), stream=st)

    def check(self) -> None:
        st = self.status.tolist()
        if st[0] != 0:
            raise TimeoutError("multicast fan-out wait timed out")
        if st[1] != 0:
            raise IndexError("multicast fan-out skipped out-of-range block ids")


class ReplicatedDataWorker:
    """Rank 0 onboards from its G2/G3, then replicates to all ranks."""

    def __init__(self, worker, collectives: CollectiveOps):
        self.worker, self.coll = worker, collectives

    def onboard(self, g2_ids: list[int] | None, g1_ids: list[int], stream=None) -> None:
        from ..logical.manager import Tier

        if self.coll.rank == 0 and g2_ids:
            self.worker.execute_local_transfer(Tier.G2, g2_ids, Tier.G1, g1_ids).wait()
        self.coll.broadcast(g1_ids, g1_ids, stream=stream)
