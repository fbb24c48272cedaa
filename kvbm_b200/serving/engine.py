"""A small serving engine that drives the block manager through its connector.

It plays the part a serving framework (vLLM) plays for the reference: a
scheduler with waiting / waiting-for-remote-KV / running requests, a G1
block allocator over one KV pool, prefill chunks under a token budget, a
static decode batch replayed as one CUDA graph per step - and, around every
step, the connector hooks in the order vLLM's v1 engine calls them:

scheduler side
    ``get_num_new_matched_tokens`` and ``update_state_after_alloc`` when a
    request is admitted, ``build_connector_meta`` once per step,
    ``update_connector_output`` with the workers' reports, and
    ``request_finished`` when a request ends (blocks stay allocated while the
    connector reports a transfer still reading them);
worker side
    ``bind_connector_metadata``, ``start_load_kv``, ``wait_for_layer_load`` /
    ``save_kv_layer`` around every layer, ``wait_for_save``,
    ``get_finished``, ``build_connector_worker_meta``,
    ``get_block_ids_with_load_errors``.

Requests whose prompt arrives from outside (a G2/G3 onboard or a remote
prefill) wait until the connector reports them received; on a full-prompt
hit the last prompt token is recomputed to sample the first output token
(vLLM's rule, v1/core/sched/scheduler.py ``_update_waiting_for_remote_kv``),
which the decode batch does as its first step for that request. Blocks
reported as failed to load are recomputed by a local prefill.

The model is ``models.llama.LlamaModel`` (random-init weights); inference
only, no sampling beyond greedy argmax, no stop tokens (requests end after
``max_tokens``).
"""

from __future__ import annotations

import enum
import math
from collections import deque
from dataclasses import dataclass, field

import torch

from ..connector.leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
from ..connector.worker import ConnectorWorker
from ..logical.manager import BlockManager, MutableBlock, Tier
from ..logical.sequence import sequence_hashes
from ..models.llama import LlamaModel
from ..ops import llama_ops
from ..physical.layout import KvLayout


class RequestStatus(str, enum.Enum):
    WAITING = "waiting"
    WAITING_FOR_REMOTE_KVS = "waiting_for_remote_kvs"
    PREFILL = "prefill"
    DECODE = "decode"
    FINISHED = "finished"


@dataclass
class Request:
    request_id: str
    prompt: torch.Tensor                 # int32 [S] on the host (pinned for an asynchronous upload)
    max_tokens: int = 1
    kv_transfer_params: dict | None = None
    salt: str | None = None
    status: RequestStatus = RequestStatus.WAITING
    num_computed_tokens: int = 0
    num_cached_tokens: int = 0           # prompt tokens found in this engine's own G1 prefix cache
    num_external_tokens: int = 0         # prompt tokens the connector loads (G2/G3 onboard or a remote prefill)
    block_ids: list[int] = field(default_factory=list)
    num_output: int = 0
    slot: int = -1
    output: torch.Tensor | None = None   # pinned int64 [max_tokens]; valid once the engine's stream passed the step
    arrival_event: torch.cuda.Event | None = None
    first_token_event: torch.cuda.Event | None = None
    finish_event: torch.cuda.Event | None = None
    load_failed: bool = False
    _dev_prompt: torch.Tensor | None = None
    _dev_ids: torch.Tensor | None = None
    _first_tok: torch.Tensor | None = None
    _handles: list = field(default_factory=list)   # prefix-cache mode: G1 block handles held
    _hashes: list[int] | None = None

    @property
    def num_prompt_tokens(self) -> int:
        return int(self.prompt.numel())


@dataclass
class EngineConfig:
    num_gpu_blocks: int
    block_size: int = 16
    max_num_seqs: int = 32               # decode batch slots
    max_num_batched_tokens: int = 8192   # prefill tokens per step
    max_model_len: int = 16384
    max_tokens: int = 256                # largest max_tokens a request may ask for (sizes the output buffer)
    use_graphs: bool = True
    decode_splits: int | None = None
    record_events: bool = True           # arrival / first-token CUDA events per request
    max_inflight_steps: int = 2          # the host runs at most this many steps ahead of the GPU
    prefix_caching: bool = False         # keep finished prompts' full blocks in G1 (LRU) and match them first


class DecodeBatch:
    """``slots`` decode sequences with static shapes; one step is one CUDA graph replay.

    Idle slots point at block 0 (reserved by the engine) at position 0 and
    compute a throw-away token; a slot's position, length and output index
    advance only while it is active.
    """

    def __init__(self, model: LlamaModel, pool: KvLayout, slots: int, max_blocks: int, max_out: int, splits: int,
                 use_graphs: bool = True, dummy_block: int = 0):
        self.model, self.pool, self.slots = model, pool, slots
        self.dummy = int(dummy_block)
        self.max_blocks, self.max_out, self.splits = max_blocks, max_out, splits
        dev = model.device
        self.tok = torch.zeros(slots, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.seq_lens = torch.ones(slots, dtype=torch.int32, device=dev)
        self.block_table = torch.full((slots, max_blocks), self.dummy, dtype=torch.int32, device=dev)
        self.active = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.out_idx = torch.zeros(slots, 1, dtype=torch.int64, device=dev)
        self.out = torch.zeros(slots, max_out, dtype=torch.int64, device=dev)
        self.use_graphs = use_graphs
        self.graph: torch.cuda.CUDAGraph | None = None
        self.graph_launches = 0

    def _step(self) -> None:
        nxt = self.model.decode_step(self.tok, self.pos, self.pool, self.block_table, self.seq_lens, self.splits)
        self.out.scatter_(1, self.out_idx, nxt.unsqueeze(1))
        self.tok.copy_(nxt)
        self.pos.add_(self.active)
        self.seq_lens.add_(self.active)
        self.out_idx.add_(self.active.unsqueeze(1))
        self.out_idx.clamp_(max=self.max_out - 1)

    def _reset(self) -> None:
        self.tok.zero_()
        self.pos.zero_()
        self.seq_lens.fill_(1)
        self.block_table.fill_(self.dummy)
        self.active.zero_()
        self.out_idx.zero_()

    def capture(self) -> None:
        if not self.use_graphs or self.graph is not None:
            return
        from ..ops import _lib

        s = torch.cuda.Stream(device=self.model.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        before = _lib.launch_count()
        with torch.cuda.graph(g):
            self._step()
        self.graph_launches = _lib.launch_count() - before
        self.graph = g
        self._reset()

    def enter(self, entries: list[tuple[int, list[int], int, int, int]]) -> None:
        """Activate slots: ``(slot, block_ids, input_token, position, first_output_index)`` each.
        ``input_token < 0`` keeps the token already in the slot (written by the caller)."""
        if not entries:
            return
        n = len(entries)
        dev = self.tok.device
        slots = torch.tensor([e[0] for e in entries], dtype=torch.int64)
        rows = torch.full((n, self.max_blocks), self.dummy, dtype=torch.int32)
        for i, e in enumerate(entries):
            if len(e[1]) > self.max_blocks:
                raise ValueError(f"{len(e[1])} blocks exceed the decode batch's {self.max_blocks}")
            rows[i, : len(e[1])] = torch.tensor(e[1], dtype=torch.int32)
        scal = torch.tensor([[e[2], e[3], e[3] + 1, e[4]] for e in entries], dtype=torch.int64)
        slots_d = slots.pin_memory().to(dev, non_blocking=True)
        rows_d = rows.pin_memory().to(dev, non_blocking=True)
        scal_d = scal.pin_memory().to(dev, non_blocking=True)
        self.block_table.index_copy_(0, slots_d, rows_d)
        keep = scal_d[:, 0] < 0
        self.tok.index_copy_(0, slots_d, torch.where(keep, self.tok.index_select(0, slots_d), scal_d[:, 0]))
        self.pos.index_copy_(0, slots_d, scal_d[:, 1].to(torch.int32))
        self.seq_lens.index_copy_(0, slots_d, scal_d[:, 2].to(torch.int32))
        self.out_idx.index_copy_(0, slots_d, scal_d[:, 3:4])
        self.active.index_fill_(0, slots_d, 1)

    def leave(self, slots: list[int]) -> None:
        if not slots:
            return
        idx = torch.tensor(slots, dtype=torch.int64).pin_memory().to(self.tok.device, non_blocking=True)
        self.active.index_fill_(0, idx, 0)
        self.pos.index_fill_(0, idx, 0)
        self.seq_lens.index_fill_(0, idx, 1)
        self.out_idx.index_fill_(0, idx, 0)
        self.block_table.index_fill_(0, idx, self.dummy)

    def step(self) -> None:
        if self.graph is not None:
            from ..ops import _lib

            self.graph.replay()
            _lib.count_launches(self.graph_launches)
        else:
            self._step()


@dataclass
class StepPlan:
    """Everything a model runner needs to execute one engine step.

    The scheduling rank builds it; with tensor parallelism it is broadcast so
    every rank runs the same prefill chunks and decode step on its shard (the
    collectives inside the forward pass line up) and the same connector ops on
    its KV shard."""

    step: int
    meta: bytes | None = None
    new: list[tuple] = field(default_factory=list)        # (req_id, prompt int32 bytes, block_ids, max_tokens)
    enter: list[tuple] = field(default_factory=list)      # (slot, req_id, input token or -1, position, output index)
    prefills: list[tuple] = field(default_factory=list)   # (req_id, start, end)
    decode: bool = False
    finish: list[tuple] = field(default_factory=list)     # (req_id, slot, n tokens): decode ends after this step
    done: list[str] = field(default_factory=list)         # every request that ends in this step


class LLMEngine:
    """One serving instance with an optional block-manager connector.

    Single GPU by default. With ``tp`` (a :class:`~kvbm_b200.serving.tp.TpComm`)
    the instance spans ``tp.size`` processes: rank 0 schedules (it holds the
    connector leader and the G1 block allocator) and broadcasts each step's
    plan; every rank runs the plan on its model shard and its connector
    worker, and rank 0 aggregates the workers' reports (a request counts as
    received / sent when every rank reported it, the way vLLM aggregates its
    workers' outputs).
    """

    def __init__(self, model: LlamaModel, cfg: EngineConfig, leader: ConnectorLeader | None = None,
                 worker: ConnectorWorker | None = None, pool: KvLayout | None = None, tp=None):
        self.model, self.cfg = model, cfg
        self.device = model.device
        self.pool = pool if pool is not None else model.allocate_pool(cfg.num_gpu_blocks, cfg.block_size)
        self.tp = tp
        self.is_scheduler = tp is None or tp.rank == 0
        self.leader, self.worker = (leader if self.is_scheduler else None), worker
        self.g1: BlockManager | None = None
        if cfg.prefix_caching:
            # G1 blocks through the logical block manager: finished prompts' full blocks stay
            # registered (inactive, LRU-evicted) and later prompts match them before asking the connector
            self.g1 = BlockManager(cfg.num_gpu_blocks, cfg.block_size, "lru", Tier.G1)
            self._dummy_handle = self.g1.allocate_blocks(1)[0]  # target of idle decode slots, never freed
            dummy = self._dummy_handle.block_id
            self.free_blocks = deque()
        else:
            self.free_blocks = deque(range(1, cfg.num_gpu_blocks))  # block 0: target of idle decode slots
            dummy = 0
        self.requests: dict[str, Request] = {}
        self._mirror: dict[str, Request] = {}   # TP ranks > 0: the requests the plans named
        self.waiting: deque[Request] = deque()
        self.remote: dict[str, Request] = {}
        self.prefilling: deque[Request] = deque()
        self.ready: deque[Request] = deque()
        self.decoding: dict[int, Request] = {}
        self.free_slots = deque(range(cfg.max_num_seqs))
        self._delayed: dict[str, Request] = {}
        self._announced: set[str] = set()
        self._recv_count: dict[str, int] = {}
        self._send_count: dict[str, int] = {}
        self.step_id = 0
        self._mark = torch.cuda.Stream(device=self.device) if cfg.record_events else None
        max_blocks = math.ceil(cfg.max_model_len / cfg.block_size)
        splits = cfg.decode_splits or llama_ops.decode_splits(cfg.max_num_seqs, model.cfg.kv_heads,
                                                              cfg.max_model_len, cfg.block_size)
        self.batch = DecodeBatch(model, self.pool, cfg.max_num_seqs, max_blocks, cfg.max_tokens, splits,
                                 cfg.use_graphs, dummy_block=dummy)
        self.stats = {"steps": 0, "prefill_tokens": 0, "decode_steps": 0, "finished": 0, "recomputed": 0,
                      "prompt_tokens": 0, "g1_hit_tokens": 0, "external_tokens": 0}
        self._inflight: deque[torch.cuda.Event] = deque()

    # ------------------------------------------------------------- public
    def warmup(self) -> None:
        """Capture the decode step's CUDA graph (before the first timed step)."""
        self.batch.capture()
        torch.cuda.synchronize(self.device)

    def release_graphs(self) -> None:
        """Drop the captured decode graph. A tensor-parallel instance's graph holds NCCL
        all-reduces, and a process group cannot be destroyed while a graph that calls it
        is alive, so instances release their graphs before their groups go away."""
        torch.cuda.synchronize(self.device)
        self.batch.graph = None

    def add_request(self, req: Request) -> None:
        if not self.is_scheduler:
            raise RuntimeError("requests enter a tensor-parallel instance on its rank 0")
        if req.max_tokens > self.cfg.max_tokens:
            raise ValueError(f"max_tokens {req.max_tokens} > engine limit {self.cfg.max_tokens}")
        if req.num_prompt_tokens + req.max_tokens > self.cfg.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        self.requests[req.request_id] = req
        if self._mark is not None:
            req.arrival_event = torch.cuda.Event(enable_timing=True)
            req.arrival_event.record(self._mark)
        if self.leader is not None:
            self.leader.create_slot(KvbmRequest(req.request_id, req.prompt.tolist(), salt=req.salt,
                                                max_tokens=req.max_tokens,
                                                kv_transfer_params=req.kv_transfer_params))
        self.waiting.append(req)

    def has_unfinished(self) -> bool:
        return bool(self.requests)

    @property
    def num_waiting_for_remote(self) -> int:
        return len(self.remote)

    def step(self) -> list[Request]:
        """One engine step; returns the requests that finished in it (on the scheduling rank)."""
        self.step_id += 1
        self.stats["steps"] += 1
        self._finished_now: list[Request] = []
        plan = self._schedule() if self.is_scheduler else None
        if self.tp is not None:
            plan = self.tp.broadcast_plan(plan)
        self._execute(plan)
        report = self._report(plan)
        if self.tp is not None:
            reports = self.tp.gather_reports(report)
        else:
            reports = [report]
        if self.is_scheduler:
            self._update(reports)
        # bounded lookahead: what the connector polls reflects the GPU's progress, as in an engine that
        # reads its sampled tokens every step
        ev = torch.cuda.Event()
        ev.record()
        self._inflight.append(ev)
        while len(self._inflight) > max(1, self.cfg.max_inflight_steps):
            self._inflight.popleft().synchronize()
        return self._finished_now

    # ----------------------------------------------------------- schedule
    def _schedule(self) -> StepPlan:
        plan = StepPlan(step=self.step_id)
        so = SchedulerOutputLite(step=self.step_id)
        self._admit(so)
        for req in self.prefilling:
            if req.request_id not in self._announced:
                self._announce(req, plan)
        self._plan_prefill(so, plan)
        self._plan_enter(so, plan)
        for slot, req in self.decoding.items():
            if req.request_id not in so.scheduled:
                so.scheduled[req.request_id] = ([], [], req.num_prompt_tokens + req.num_output)
            if req.num_output + 1 >= req.max_tokens:
                plan.finish.append((req.request_id, slot, req.max_tokens))
        plan.decode = bool(self.decoding)
        plan.done = [rid for rid, _, _ in plan.finish]
        plan.done += [rid for rid, _, end in plan.prefills
                      if end >= self.requests[rid].num_prompt_tokens and self.requests[rid].max_tokens <= 1]
        if self.leader is not None:
            plan.meta = self.leader.build_connector_meta(so)
        return plan

    def _announce(self, req: Request, plan: StepPlan) -> None:
        """Tell the other TP ranks about a request the first time a plan uses it."""
        self._announced.add(req.request_id)
        if self.tp is not None:
            plan.new.append((req.request_id, req.prompt.numpy().tobytes(), list(req.block_ids), req.max_tokens))

    def _blocks_needed(self, req: Request) -> int:
        return math.ceil((req.num_prompt_tokens + max(0, req.max_tokens - 1)) / self.cfg.block_size)

    def _allocate(self, req: Request, need: int) -> bool:
        """G1 blocks for ``req`` (its cached prefix first in prefix-cache mode); False if G1 is full."""
        if self.g1 is None:
            if len(self.free_blocks) < need:
                return False
            req.block_ids = [self.free_blocks.popleft() for _ in range(need)]
            req.num_cached_tokens = 0
            return True
        bs = self.cfg.block_size
        if req._hashes is None:
            req._hashes = sequence_hashes(req.prompt.numpy(), bs, req.salt)
        hits = self.g1.match_blocks(req._hashes[: (req.num_prompt_tokens - 1) // bs])
        fresh = self.g1.allocate_blocks(need - len(hits))
        if fresh is None:
            for b in hits:
                b.release()
            return False
        req._handles = hits + fresh
        req.block_ids = [b.block_id for b in req._handles]
        req.num_cached_tokens = len(hits) * bs
        return True

    def _register_prompt(self, req: Request) -> None:
        """Prefix-cache mode: the prompt's full blocks hold their final K/V now; make them matchable."""
        if self.g1 is None or not req._handles:
            return
        nfull = req.num_prompt_tokens // self.cfg.block_size
        first = req.num_cached_tokens // self.cfg.block_size
        fresh = [b for b in req._handles[first:nfull] if isinstance(b, MutableBlock)]
        if len(fresh) != nfull - first:
            return  # already registered
        reg = self.g1.register_mutable(fresh, req._hashes[first:nfull])
        req._handles = req._handles[:first] + reg + req._handles[nfull:]

    def _admit(self, so: SchedulerOutputLite) -> None:
        for _ in range(len(self.waiting)):
            req = self.waiting[0]
            need = self._blocks_needed(req)
            if not self._allocate(req, need):
                break
            n_ext, is_async = 0, False
            if self.leader is not None:
                n_ext, is_async = self.leader.get_num_new_matched_tokens(req.request_id, req.num_cached_tokens)
                if n_ext is None:  # the connector is still searching: try again next step
                    self._release_blocks(req)
                    self.waiting.rotate(-1)
                    continue
            self.waiting.popleft()
            if self.leader is not None:
                self.leader.update_state_after_alloc(req.request_id, req.block_ids, n_ext)
            req.num_external_tokens = n_ext
            self.stats["prompt_tokens"] += req.num_prompt_tokens
            self.stats["g1_hit_tokens"] += req.num_cached_tokens
            self.stats["external_tokens"] += n_ext
            if n_ext and is_async:
                req.status = RequestStatus.WAITING_FOR_REMOTE_KVS
                req.num_computed_tokens = req.num_cached_tokens
                self.remote[req.request_id] = req
            else:
                req.num_computed_tokens = req.num_cached_tokens + n_ext
                req.status = RequestStatus.PREFILL
                self.prefilling.append(req)

    def _plan_prefill(self, so: SchedulerOutputLite, plan: StepPlan) -> None:
        budget = self.cfg.max_num_batched_tokens
        for req in self.prefilling:
            if budget <= 0:
                break
            start = req.num_computed_tokens
            end = min(req.num_prompt_tokens, start + budget)
            plan.prefills.append((req.request_id, start, end))
            budget -= end - start
            so.scheduled[req.request_id] = ([], [], end)

    def _plan_enter(self, so: SchedulerOutputLite, plan: StepPlan) -> None:
        while self.ready and self.free_slots:
            req = self.ready.popleft()
            slot = self.free_slots.popleft()
            req.slot, req.status = slot, RequestStatus.DECODE
            S = req.num_prompt_tokens
            if req.request_id not in self._announced:
                self._announce(req, plan)
            if req.num_output >= 1:
                # prefilled here: the sampled token is on the device (every rank has it), output 0 written
                plan.enter.append((slot, req.request_id, -1, S, 1))
            else:
                # every prompt token's KV arrived: the first step recomputes the last one
                plan.enter.append((slot, req.request_id, int(req.prompt[S - 1]), S - 1, 0))
                so.scheduled[req.request_id] = ([], [], S)
            self.decoding[slot] = req

    # ------------------------------------------------------------ execute
    def _req(self, rid: str) -> Request:
        req = self.requests.get(rid) or self._mirror.get(rid) or self._delayed.get(rid)
        if req is None:
            raise KeyError(f"plan names unknown request {rid}")
        return req

    def _execute(self, plan: StepPlan) -> None:
        for rid, prompt, block_ids, max_tokens in plan.new:
            if not self.is_scheduler and rid not in self._mirror:
                t = torch.frombuffer(bytearray(prompt), dtype=torch.int32)
                m = Request(rid, t, max_tokens=max_tokens)
                m.block_ids = list(block_ids)
                self._mirror[rid] = m
        w = self.worker
        if w is not None and plan.meta is not None:
            w.bind_connector_metadata(plan.meta)
            w.start_load_kv()
        entries = []
        for slot, rid, tok, pos, oi in plan.enter:
            req = self._req(rid)
            if tok < 0:
                self.batch.tok[slot: slot + 1].copy_(req._first_tok)
                self.batch.out[slot, 0:1].copy_(req._first_tok)
                req._first_tok = None
            entries.append((slot, req.block_ids, tok, pos, oi))
        self.batch.enter(entries)
        for rid, start, end in plan.prefills:
            self._run_prefill(self._req(rid), start, end)
        if plan.decode:
            self.batch.step()
            self.stats["decode_steps"] += 1
            leave = []
            for rid, slot, n in plan.finish:
                if self.is_scheduler:
                    req = self._req(rid)
                    req.output = torch.empty(n, dtype=torch.int64, pin_memory=self.device.type == "cuda")
                    req.output.copy_(self.batch.out[slot, :n], non_blocking=True)
                else:
                    self._mirror.pop(rid, None)
                leave.append(slot)
            self.batch.leave(leave)
            if self.is_scheduler:
                self._advance_decode(plan)
        if w is not None and plan.meta is not None:
            w.wait_for_save()

    def _run_prefill(self, req: Request, start: int, end: int) -> None:
        dev = self.device
        if req._dev_prompt is None:
            p = req.prompt if req.prompt.is_pinned() else req.prompt.pin_memory()
            req._dev_prompt = p.to(dev, non_blocking=True)
            req._dev_ids = torch.tensor(req.block_ids, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        w = self.worker
        rid = {req.request_id}
        nxt = self.model.prefill(req._dev_prompt[start:end], self.pool, req._dev_ids, start_pos=start,
                                 on_layer_done=(lambda l: w.save_kv_layer(l, requests=rid)) if w else None,
                                 on_layer_start=w.wait_for_layer_load if w else None)
        self.stats["prefill_tokens"] += end - start
        if end < req.num_prompt_tokens:
            if self.is_scheduler:
                req.num_computed_tokens = end
            return
        if not self.is_scheduler:
            if req.max_tokens > 1:
                req._first_tok = nxt
            else:
                self._mirror.pop(req.request_id, None)
            return
        req.num_computed_tokens = end
        self.prefilling.remove(req)
        self._register_prompt(req)
        req.num_output = 1
        if self._mark is not None:
            req.first_token_event = torch.cuda.Event(enable_timing=True)
            req.first_token_event.record()
        if req.max_tokens <= 1:
            req.output = torch.empty(1, dtype=torch.int64, pin_memory=self.device.type == "cuda")
            req.output.copy_(nxt, non_blocking=True)
            self._finish(req)
        else:
            req._first_tok = nxt
            self.ready.append(req)

    def _advance_decode(self, plan: StepPlan) -> None:
        ev = None
        ending = {rid for rid, _, _ in plan.finish}
        for slot, req in list(self.decoding.items()):
            req.num_output += 1
            if self._mark is not None and (req.num_output == 1 or req.request_id in ending):
                if ev is None:
                    ev = torch.cuda.Event(enable_timing=True)
                    ev.record()
                if req.num_output == 1:
                    req.first_token_event = ev
                if req.request_id in ending:
                    req.finish_event = ev
            if req.request_id in ending:
                del self.decoding[slot]
                self.free_slots.append(slot)
                self._finish(req)

    # ------------------------------------------------------------- report
    def _report(self, plan: StepPlan) -> dict:
        """This rank's connector-worker outputs for the step."""
        w = self.worker
        if w is None:
            return {}
        sending, recving = w.get_finished(set(plan.done))
        out = {"sending": sending, "recving": recving, "meta": w.build_connector_worker_meta(),
               "errors": w.get_block_ids_with_load_errors()}
        w.clear_connector_metadata()
        return out

    def _update(self, reports: list[dict]) -> None:
        if self.leader is None:
            return
        n = len(reports)
        sending, recving, errs, meta = set(), set(), set(), {}
        for rep in reports:
            for r in rep.get("sending", ()):
                self._send_count[r] = self._send_count.get(r, 0) + 1
            for r in rep.get("recving", ()):
                self._recv_count[r] = self._recv_count.get(r, 0) + 1
            errs |= set(rep.get("errors", ()))
            for kind, steps in (rep.get("meta") or {}).items():
                d = meta.setdefault(kind, {})
                for st, c in steps.items():
                    d[st] = d.get(st, 0) + c
        for r, c in list(self._send_count.items()):
            if c >= n:
                sending.add(r)
                del self._send_count[r]
        for r, c in list(self._recv_count.items()):
            if c >= n:
                recving.add(r)
                del self._recv_count[r]
        self.leader.update_connector_output(sending, recving, meta or None, errs)
        self._on_received(recving, errs)
        self._on_sent(sending)

    # -------------------------------------------------------- completion
    def _finish(self, req: Request) -> None:
        self._finished_now.append(req)
        req.status = RequestStatus.FINISHED
        self.requests.pop(req.request_id, None)
        self.stats["finished"] += 1
        delay = False
        if self.leader is not None:
            delay, _ = self.leader.request_finished(req.request_id, req.block_ids)
        if delay:
            self._delayed[req.request_id] = req
        else:
            self._free(req)

    def _free(self, req: Request) -> None:
        # the request keeps the list of the blocks it held (for inspection); the blocks return to the pool
        self._release_blocks(req)
        self._announced.discard(req.request_id)

    def _release_blocks(self, req: Request) -> None:
        if self.g1 is None:
            self.free_blocks.extend(req.block_ids)
            return
        for b in req._handles:
            b.release()  # registered blocks stay cached (inactive) until G1 evicts them
        req._handles = []

    def _on_sent(self, sending: set[str]) -> None:
        for rid in sending:
            req = self._delayed.pop(rid, None)
            if req is not None:
                self._free(req)

    def _on_received(self, recving: set[str], errs: set[int]) -> None:
        for rid in recving:
            req = self.remote.pop(rid, None)
            if req is None:
                continue
            S = req.num_prompt_tokens
            if errs and errs.intersection(req.block_ids):
                # the external KV never arrived: recompute the prompt here
                req.load_failed = True
                req.num_computed_tokens = req.num_cached_tokens
                req.status = RequestStatus.PREFILL
                self.prefilling.append(req)
                self.stats["recomputed"] += 1
                continue
            req.num_computed_tokens = req.num_cached_tokens + req.num_external_tokens
            if req.num_computed_tokens >= S and req.max_tokens > 1:
                req.num_computed_tokens = S - 1
                self._register_prompt(req)
                self.ready.append(req)
            else:
                req.num_computed_tokens = min(req.num_computed_tokens, S - 1)
                req.status = RequestStatus.PREFILL
                self.prefilling.append(req)
