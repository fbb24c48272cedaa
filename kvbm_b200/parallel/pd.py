"""Prefill -> decode KV transfer over NVLink (one box, one process per GPU).

The decode instance exports, through CUDA IPC, its paged G1 KV pool and a
small "mailbox" page (one completion flag + payload words per request slot).
The prefill instance maps both and, for every finished prefill layer, launches
one fused transfer kernel on a side stream that gathers the layer's paged
blocks from its own pool, applies the layout transform / KV-head reshard /
fp8 quantisation the two pools need, and stores straight into the decode
pool's blocks over NVLink. After the last layer of a request a one-thread
kernel copies the payload (the first generated token) into the mailbox and
release-stores the slot's flag at system scope. The decode instance waits on
the flags with a bounded-spin kernel on its own stream, so no NCCL/NIXL call
and no host round trip sits on the data path.

When prefill and decode share a GPU (colocated) the same kernels write the
local pool and completion is a CUDA event instead of a flag.

Parity: replaces the reference's pull of prefill G2 blocks over NIXL
(crates/kvbm-engine/src/leader/instance.rs:1394 rdma_pull_with_opts ->
plan_pull G2->G2) followed by a G2->G1 onboard; head-slicing follows
crates/kvbm-engine/src/p2p/dispatch.rs:17-47.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import kv_ops
from ..physical.layout import KvLayout, LayoutDescriptor
from ..physical.memory import DeviceBuffer, PeerBuffer

WAIT_TIMEOUT_NS = 30_000_000_000  # 30 s: far above any transfer, bounds a dead peer


@dataclass
class MailboxDescriptor:
    handle: bytes
    slots: int
    nbytes: int


class Mailbox:
    """Decode-side flags + payload words, one slot per in-flight request."""

    PAYLOAD_WORDS = 1

    def __init__(self, slots: int, device: int | None = None):
        self.slots = slots
        nbytes = slots * 8 * (1 + self.PAYLOAD_WORDS) + 256
        self.buf = DeviceBuffer(nbytes, device=device, zero=True)
        self.flags = self.buf.ptr
        self.payload = self.buf.ptr + slots * 8
        self.status = self.buf.ptr + slots * 8 * (1 + self.PAYLOAD_WORDS)
        t = self.buf.tensor(torch.uint8)
        self.flags_t = t[: slots * 8].view(torch.int64)
        self.payload_t = t[slots * 8: slots * 8 * 2].view(torch.int64)
        self.status_t = t[slots * 16: slots * 16 + 4].view(torch.int32)

    def descriptor(self) -> MailboxDescriptor:
        return MailboxDescriptor(self.buf.ipc_handle(), self.slots, self.buf.nbytes)

    def wait_all(self, n: int, seq: int, stream=None, timeout_ns: int = WAIT_TIMEOUT_NS) -> None:
        kv_ops.wait_flags_all(self.flags, n, seq, timeout_ns, self.status, stream=stream)

    def check(self) -> None:
        """Raise if a bounded wait gave up (call after synchronizing the stream)."""
        st = int(self.status_t.item())
        if st != 0:
            raise TimeoutError(f"P->D completion wait timed out (status {st}); peer dead or stalled")


class PdSender:
    """Prefill-side end of one P->D channel."""

    def __init__(self, local_pool: KvLayout, remote_pool: KvLayout, mailbox: PeerBuffer | None,
                 mailbox_slots: int = 0, engine: str = "tma", max_ctas: int = 0, stream: torch.cuda.Stream | None = None,
                 timing: bool = True):
        self.local = local_pool
        self.remote = remote_pool
        self.mailbox = mailbox
        self.slots = mailbox_slots
        self.engine = engine
        self.max_ctas = max_ctas
        # highest priority: transfer CTAs are scheduled ahead of queued prefill CTAs
        self.stream = stream or torch.cuda.Stream(priority=-100)
        self.timing = timing
        self._timers: list[tuple[torch.cuda.Event, torch.cuda.Event, int]] = []
        self.bytes_per_layer_block = local_pool.config.outer_dim * local_pool.config.bytes_per_chunk

    @classmethod
    def connect(cls, local_pool: KvLayout, pool_desc: LayoutDescriptor, mailbox_desc: MailboxDescriptor | None,
                **kw) -> "PdSender":
        remote = KvLayout.from_descriptor(pool_desc)
        mb = PeerBuffer(mailbox_desc.handle, mailbox_desc.nbytes) if mailbox_desc else None
        return cls(local_pool, remote, mb, mailbox_desc.slots if mailbox_desc else 0, **kw)

    def send_layer(self, layer: int, src_ids: torch.Tensor, dst_ids: torch.Tensor,
                   after: torch.cuda.Stream | None = None, num_layers: int = 1, src_head_offset: int = 0,
                   dst_head_offset: int = 0, num_heads: int | None = None,
                   on_stream: torch.cuda.Stream | None = None) -> None:
        """Transfer ``num_layers`` layers starting at ``layer`` once ``after``'s queued work is done.

        By default the copy runs on this sender's high-priority side stream,
        overlapping whatever ``after`` does next (and competing with it for
        SMs). With ``on_stream`` it runs in that stream's order instead (the
        prefill stream, between the layer's KV write and the next GEMM), so
        it has the GPU to itself.
        """
        st = on_stream if on_stream is not None else self.stream
        if after is not None and on_stream is None:
            self.stream.wait_stream(after)
        with torch.cuda.stream(st):
            if self.timing:
                s = torch.cuda.Event(enable_timing=True)
                e = torch.cuda.Event(enable_timing=True)
                s.record(st)
            kv_ops.kv_transfer(self.local, src_ids, self.remote, dst_ids, layer_begin=layer, num_layers=num_layers,
                               src_head_offset=src_head_offset, dst_head_offset=dst_head_offset,
                               num_heads=num_heads, engine=self.engine.removesuffix("_inline"),
                               max_ctas=self.max_ctas, stream=st)
            if self.timing:
                e.record(st)
                nbytes = len(src_ids) * num_layers * self.bytes_per_layer_block
                self._timers.append((s, e, nbytes))

    def complete(self, slot: int, seq: int, payload: torch.Tensor | None = None) -> torch.cuda.Event:
        """Publish request ``slot`` as delivered (flag = seq) after its transfers."""
        ev = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            if self.mailbox is not None:
                flag = self.mailbox.ptr + slot * 8
                if payload is not None:
                    dst = self.mailbox.ptr + self.slots * 8 + slot * 8
                    kv_ops.signal_flag_payload(flag, seq, dst, payload.data_ptr(), 1, stream=self.stream)
                else:
                    kv_ops.signal_flag(flag, seq, stream=self.stream)
            ev.record(self.stream)
        return ev

    def take_timings(self) -> tuple[float, int]:
        """(total transfer-kernel ms, total bytes) since the last call. Synchronizes the stream."""
        self.stream.synchronize()
        ms = sum(s.elapsed_time(e) for s, e, _ in self._timers)
        nb = sum(b for _, _, b in self._timers)
        self._timers.clear()
        return ms, nb
