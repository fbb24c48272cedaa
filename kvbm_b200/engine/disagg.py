"""Disaggregated prefill/decode serving on one box: the public API the
benchmarks drive.

A *wave* is ``concurrency`` requests that arrive together at one decode
instance: the paired prefill instance prefills them one after another,
streaming every finished layer's KV straight into the decode instance's
paged G1 pool (``parallel.pd``), and hands over the first generated token
with the completion flag; the decode instance then generates the remaining
tokens for the whole batch with a CUDA-graph-captured decode step.

``DisaggServer.serve_wave(prompts)`` takes pinned host prompts and returns
host output tokens, so one call covers the H2D copy of the step's inputs,
prefill, the P->D transfer, decode and the D2H read of the results.

Roles follow the reference's conditional-disaggregation flow
(crates/kvbm-engine/src/remote/cd/*, docs/conditional-pd.md): the decode
side owns the destination blocks (it allocates them in its G1 block pool and
sends their ids with the request), the prefill side produces the first token
and makes the blocks available. The data path is the fused NVLink kernel
instead of NIXL through pinned host memory.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .. import _core_native as core
from ..models.llama import KvPush, LlamaConfig, LlamaModel
from ..ops import llama_ops
from ..ops import kv_ops
from ..parallel.pd import WAIT_TIMEOUT_NS, Mailbox, PdSender
from ..physical.layout import LayoutDescriptor


@dataclass
class DisaggConfig:
    model: LlamaConfig = field(default_factory=LlamaConfig.llama3_8b)
    concurrency: int = 32
    prompt_len: int = 8192
    gen_len: int = 256
    page_size: int = 16
    engine: str = "fused"  # fused (RoPE/KV kernel pushes) | tma | tile (side-stream copy) | tma_inline | tile_inline
    max_ctas: int = 0
    layer_batch: int = 1   # copy engines: layers moved per transfer launch (fused pushes every layer)
    prefill_buffers: int = 2
    decode_splits: int | None = None
    use_graphs: bool = True
    seed: int = 0

    @property
    def prompt_blocks(self) -> int:
        return math.ceil(self.prompt_len / self.page_size)

    @property
    def request_blocks(self) -> int:
        return math.ceil((self.prompt_len + self.gen_len) / self.page_size)

    def kv_bytes_per_request(self) -> int:
        c = self.model
        return self.prompt_blocks * c.layers * 2 * self.page_size * c.kv_heads * c.head_dim * 2


class DecodeInstance:
    """Decode side: G1 pool + block pool, mailbox, graph-captured decode step.

    With ``buffers=2`` two waves can be in flight: wave k+1's destination
    blocks are allocated and dispatched to prefill before wave k is decoded,
    so prefill of k+1 overlaps decode of k on the other GPU.
    """

    def __init__(self, model: LlamaModel, cfg: DisaggConfig, buffers: int = 1):
        self.model, self.cfg = model, cfg
        C, bpr = cfg.concurrency, cfg.request_blocks
        self.buffers = buffers
        self.num_blocks = buffers * C * bpr + 1
        self.pool = model.allocate_pool(self.num_blocks, cfg.page_size)
        self.blocks = core.BlockPool(self.num_blocks, cfg.page_size, "lru", 0)
        self.mailbox = Mailbox(buffers * C, device=model.device.index)
        dev = model.device
        self.block_table = torch.zeros(C, bpr, dtype=torch.int32, device=dev)
        self.tables = [torch.zeros(C, bpr, dtype=torch.int32, device=dev) for _ in range(buffers)]
        self.tok = torch.zeros(C, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(C, dtype=torch.int32, device=dev)
        self.seq_lens = torch.zeros(C, dtype=torch.int32, device=dev)
        self.step_idx = torch.zeros(C, 1, dtype=torch.int64, device=dev)
        self.tokens_out = torch.zeros(C, cfg.gen_len, dtype=torch.int64, device=dev)
        self.splits = cfg.decode_splits or llama_ops.decode_splits(C, model.cfg.kv_heads,
                                                                    cfg.prompt_len + cfg.gen_len, cfg.page_size)
        self.graph: torch.cuda.CUDAGraph | None = None
        self._ids: list[list[int]] = [[] for _ in range(buffers)]
        self.graph_launches = 0

    def begin_wave(self, buf: int = 0) -> torch.Tensor:
        """Allocate destination blocks for every request of wave buffer ``buf``;
        returns the [C, blocks] id table (CPU)."""
        C, bpr = self.cfg.concurrency, self.cfg.request_blocks
        got = self.blocks.allocate(C * bpr)
        if got is None:
            raise RuntimeError("decode pool exhausted")
        self._ids[buf] = got[0]
        table = torch.tensor(self._ids[buf], dtype=torch.int32).view(C, bpr)
        self.tables[buf].copy_(table)
        return table

    def end_wave(self, buf: int = 0) -> None:
        self.blocks.release_mutable_many(self._ids[buf])
        self._ids[buf] = []

    def _step(self) -> None:
        nxt = self.model.decode_step(self.tok, self.pos, self.pool, self.block_table, self.seq_lens, self.splits)
        self.tok.copy_(nxt)
        self.pos.add_(1)
        self.seq_lens.add_(1)
        self.step_idx.add_(1)
        self.tokens_out.scatter_(1, self.step_idx, self.tok.unsqueeze(1))

    def capture(self) -> None:
        """Capture one decode step as a CUDA graph (static buffers)."""
        if not self.cfg.use_graphs or self.graph is not None:
            return
        from ..ops import _lib

        self.pos.fill_(self.cfg.prompt_len)
        self.seq_lens.fill_(self.cfg.prompt_len + 1)
        self.step_idx.zero_()
        s = torch.cuda.Stream(device=self.model.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self.step_idx.zero_()
                self._step()
        torch.cuda.current_stream().wait_stream(s)
        self.step_idx.zero_()
        g = torch.cuda.CUDAGraph()
        before = _lib.launch_count()
        with torch.cuda.graph(g):
            self._step()
        self.graph_launches = _lib.launch_count() - before
        self.graph = g

    def decode(self, seq: int, stream: torch.cuda.Stream, buf: int = 0) -> tuple[torch.cuda.Event, torch.cuda.Event]:
        """Wait for every request's KV + first token, then generate. Returns (start, end) events."""
        from ..ops import _lib

        C, cfg = self.cfg.concurrency, self.cfg
        base = buf * C
        with torch.cuda.stream(stream):
            kv_ops.wait_flags_all(self.mailbox.flags + base * 8, C, seq, WAIT_TIMEOUT_NS, self.mailbox.status,
                                  stream=stream)
            start = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            self.block_table.copy_(self.tables[buf])
            self.tok.copy_(self.mailbox.payload_t[base: base + C])
            self.pos.fill_(cfg.prompt_len)
            self.seq_lens.fill_(cfg.prompt_len + 1)
            self.step_idx.zero_()
            self.tokens_out[:, 0].copy_(self.tok)
            for _ in range(cfg.gen_len - 1):
                if self.graph is not None:
                    self.graph.replay()
                    _lib.count_launches(self.graph_launches)
                else:
                    self._step()
            end = torch.cuda.Event(enable_timing=True)
            end.record(stream)
        return start, end


class PrefillInstance:
    """Prefill side: staging G1 pool reused across requests, first-token payloads."""

    def __init__(self, model: LlamaModel, cfg: DisaggConfig):
        self.model, self.cfg = model, cfg
        nb = cfg.prefill_buffers * cfg.prompt_blocks
        self.pool = model.allocate_pool(nb, cfg.page_size)
        self.blocks = core.BlockPool(nb, cfg.page_size, "lru", 0)
        got = self.blocks.allocate(nb)
        ids = torch.tensor(got[0], dtype=torch.int32).view(cfg.prefill_buffers, cfg.prompt_blocks)
        self.slot_ids = [ids[i].to(model.device) for i in range(cfg.prefill_buffers)]
        self.first_tok = torch.zeros(cfg.concurrency, dtype=torch.int64, device=model.device)

    def prefill_wave(self, prompts: torch.Tensor, dst_table: torch.Tensor, seq: int, sender: PdSender,
                     stream: torch.cuda.Stream, slot_base: int = 0) -> list[torch.cuda.Event]:
        """Prefill every request, streaming KV layer by layer; returns per-request delivery events."""
        cfg = self.cfg
        done: list[torch.cuda.Event] = []
        nbuf = cfg.prefill_buffers
        with torch.cuda.stream(stream):
            for r in range(prompts.shape[0]):
                if r >= nbuf:
                    stream.wait_event(done[r - nbuf])  # staging blocks free once delivered
                src_ids = self.slot_ids[r % nbuf]
                dst_ids = dst_table[r, : cfg.prompt_blocks]
                if sender.engine == "fused":
                    # the RoPE/KV kernel of every layer stores straight into the decode pool
                    push = KvPush(sender.remote, dst_ids, timers=sender._timers if sender.timing else None)
                    nxt = self.model.prefill(prompts[r], self.pool, src_ids, kv_push=push)
                else:
                    inline = sender.engine.endswith("_inline")
                    nl, lb = self.model.cfg.layers, max(1, cfg.layer_batch)

                    def done_layer(l, s=src_ids, d=dst_ids, inline=inline, nl=nl, lb=lb):
                        # one copy launch per batch of lb layers, issued when its last layer is written;
                        # inline: in the prefill stream (alone on the GPU), else on the side stream
                        if (l + 1) % lb and l != nl - 1:
                            return
                        first = l - (l % lb)
                        if inline:
                            sender.send_layer(first, s, d, num_layers=l + 1 - first, on_stream=stream)
                        else:
                            sender.send_layer(first, s, d, num_layers=l + 1 - first, after=stream)

                    nxt = self.model.prefill(prompts[r], self.pool, src_ids, on_layer_done=done_layer)
                self.first_tok[r: r + 1].copy_(nxt)
                sender.stream.wait_stream(stream)
                done.append(sender.complete(slot_base + r, seq, payload=self.first_tok[r: r + 1]))
        return done


@dataclass
class WaveResult:
    tokens: torch.Tensor | None          # [C, gen] on host (decode rank) or None
    step_ms: float                       # device time of this rank's part of the step
    kv_ms: float = 0.0                   # summed transfer-kernel time (prefill rank)
    kv_bytes: int = 0
    ttft_ms: list[float] = field(default_factory=list)
    decode_ms: float = 0.0


class DisaggServer:
    """One P/D pair (colocated on one GPU, or split over two ranks).

    Control messages (wave dispatch: sequence number, mailbox slot base and
    destination block table) go through a key-value store (the
    torch.distributed TCPStore); KV and first tokens never leave the GPUs.
    """

    def __init__(self, cfg: DisaggConfig, role: str, device: int, peer_rank: int | None = None,
                 group=None, store=None, pair_id: int = 0):
        assert role in ("colocated", "prefill", "decode")
        self.cfg, self.role = cfg, role
        self.peer, self.group, self.store, self.pair = peer_rank, group, store, pair_id
        torch.cuda.set_device(device)
        self.device = torch.device("cuda", device)
        self.model = LlamaModel(cfg.model, self.device, seed=cfg.seed)
        self.seq = 0
        self.prefill = self.decoder = self.sender = None
        if role in ("colocated", "decode"):
            self.decoder = DecodeInstance(self.model, cfg, buffers=2 if role == "decode" else 1)
        if role in ("colocated", "prefill"):
            self.prefill = PrefillInstance(self.model, cfg)
        if role == "colocated":
            self.sender = PdSender(self.prefill.pool, self.decoder.pool, None, 0, engine=cfg.engine,
                                   max_ctas=cfg.max_ctas)
        self.main = torch.cuda.Stream(device=self.device)
        self._pending: tuple[int, int] | None = None

    # ---------------------------------------------------------- set-up
    def connect(self) -> None:
        """Exchange pool / mailbox descriptors with the peer rank (CUDA IPC)."""
        if self.role == "colocated":
            return
        if self.role == "decode":
            payload = (self.decoder.pool.descriptor().to_dict(), self.decoder.mailbox.descriptor())
            dist.send_object_list([payload], dst=self.peer, group=self.group)
        else:
            obj = [None]
            dist.recv_object_list(obj, src=self.peer, group=self.group)
            pool_d, mb_d = obj[0]
            self.sender = PdSender.connect(self.prefill.pool, LayoutDescriptor.from_dict(pool_d), mb_d,
                                           engine=self.cfg.engine, max_ctas=self.cfg.max_ctas)

    def warmup_graphs(self) -> None:
        if self.decoder is not None:
            self.decoder.capture()
        torch.cuda.synchronize()

    # ----------------------------------------------------- control plane
    def _key(self, seq: int) -> str:
        return f"kvbm/pd/{self.pair}/wave/{seq}"

    def _dispatch(self) -> tuple[int, int]:
        """Decode side: allocate the next wave's blocks and hand them to prefill."""
        self.seq += 1
        seq = self.seq
        buf = seq % self.decoder.buffers
        table = self.decoder.begin_wave(buf)
        header = torch.tensor([seq, buf * self.cfg.concurrency], dtype=torch.int32)
        self.store.set(self._key(seq), torch.cat([header, table.view(-1)]).numpy().tobytes())
        return seq, buf

    def _receive(self) -> tuple[int, int, torch.Tensor]:
        """Prefill side: block until the next wave is dispatched."""
        seq = self.seq + 1
        raw = self.store.get(self._key(seq))
        self.store.delete_key(self._key(seq))
        arr = torch.frombuffer(bytearray(raw), dtype=torch.int32)
        self.seq = int(arr[0])
        return int(arr[0]), int(arr[1]), arr[2:].view(self.cfg.concurrency, self.cfg.request_blocks)

    # ----------------------------------------------------------- a wave
    def serve_wave(self, prompts_host: torch.Tensor | None, more: bool = False) -> WaveResult:
        """Serve one wave. Prefill/colocated ranks pass pinned host prompts [C, S]
        (int32); decode/colocated ranks get the host output tokens back.

        On a decode rank ``more=True`` dispatches the following wave before
        decoding this one (pipelining prefill of k+1 with decode of k)."""
        cfg = self.cfg
        C = cfg.concurrency
        st = self.main
        res = WaveResult(tokens=None, step_ms=0.0)
        t0 = torch.cuda.Event(enable_timing=True)
        done: list[torch.cuda.Event] = []
        if self.role == "prefill":
            seq, slot_base, table = self._receive()
            t0.record(st)  # the wave arrives when decode dispatches it
            with torch.cuda.stream(st):
                prompts = prompts_host.to(self.device, non_blocking=True)
                dst = table.to(self.device, non_blocking=True)
            done = self.prefill.prefill_wave(prompts, dst, seq, self.sender, st, slot_base)
            st.wait_event(done[-1])
        elif self.role == "decode":
            t0.record(st)
            if self._pending is None:
                self._pending = self._dispatch()
            seq, buf = self._pending
            self._pending = self._dispatch() if more else None
            dec_s, dec_e = self.decoder.decode(seq, st, buf)
        else:
            self.seq += 1
            seq = self.seq
            t0.record(st)
            self.decoder.begin_wave(0)
            with torch.cuda.stream(st):
                prompts = prompts_host.to(self.device, non_blocking=True)
            done = self.prefill.prefill_wave(prompts, self.decoder.tables[0], seq, self.sender, st)
            for ev in done:
                st.wait_event(ev)
            with torch.cuda.stream(st):
                # colocated: the first tokens stay local
                self.decoder.mailbox.payload_t[:C].copy_(self.prefill.first_tok)
                self.decoder.mailbox.flags_t[:C].fill_(seq)
            dec_s, dec_e = self.decoder.decode(seq, st, 0)
            buf = 0
        if self.decoder is not None:
            with torch.cuda.stream(st):
                out = torch.empty(C, cfg.gen_len, dtype=torch.int64, pin_memory=True)
                out.copy_(self.decoder.tokens_out, non_blocking=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t1.record(st)
        t1.synchronize()
        res.step_ms = t0.elapsed_time(t1)
        if self.decoder is not None:
            self.decoder.mailbox.check()
            res.tokens = out
            res.decode_ms = dec_s.elapsed_time(dec_e)
            self.decoder.end_wave(buf)
        if self.prefill is not None:
            for ev in done:
                ev.synchronize()
            res.ttft_ms = [t0.elapsed_time(ev) for ev in done]
            res.kv_ms, res.kv_bytes = self.sender.take_timings()
        return res
