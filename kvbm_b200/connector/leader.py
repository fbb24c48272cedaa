"""Scheduler-side connector: per-request slots over the InstanceLeader.

Hooks (called by the serving framework's scheduler, one process):

* ``get_num_new_matched_tokens(req_id, num_computed_tokens)`` - how many
  tokens beyond the framework's own G1 prefix hit can be loaded from
  outside: G2/G3 prefix matches (held by the slot), and - with conditional
  disaggregation on a decode instance - the rest of the prompt when the
  policy sends its prefill to a prefill instance (an asynchronous load);
* ``update_state_after_alloc(req_id, block_ids, num_external_tokens)`` -
  records the G1 destinations, queues the G2 -> G1 onboard and, for a
  remote prefill, dispatches the request (tokens, ``RemotePrefillParams``,
  destination block ids, mailbox slot) to the prefill instance and tells the
  workers to watch for it;
* ``build_connector_meta(scheduler_output)`` - advances every scheduled
  request's save cursor (blocks that became complete get G2 slots and are
  queued as G1 -> G2 offloads; they are registered in G2 only once every
  worker reports the copy done) and, on a prefill instance, every remote
  request's push cursor (blocks computed this step are pushed into the
  decode instance's G1 pool during the pass); returns the step's ops;
* ``update_connector_output(finished_sending, finished_recving, worker_meta)``
  - releases onboarded G2 references, registers G2 blocks whose copies
  landed, closes finished remote prefills (budget, mailbox slot);
* ``request_finished(req_id)`` - asks the framework to delay freeing G1
  blocks while an offload or a push still reads them.

Parity: crates/kvbm-connector/src/connector/leader/mod.rs:139-723 (Leader:
gnmt :449, usaa :462, build_connector_meta :493, request_finished :570,
update_connector_output :559), python/kvbm/vllm/connector/leader.py:50-347;
conditional disaggregation: crates/kvbm-engine/src/remote/cd/decode.rs:118
(decode-side plan in GNMT), budget.rs:16, tiering/engine/prefill.rs:97
(prefill accept), remote/cd/output.rs:85 (blocks made available as the
prefill produces them). Registration after the copy: tiering/offload/
engine.rs:123 (TransferExecutor -> register_blocks).
"""

from __future__ import annotations

import itertools
import threading
from collections import deque
from dataclasses import dataclass, field

from ..engine.cd import ConditionalDisagg, Decision, RemotePrefillParams
from ..engine.leader import InstanceLeader
from ..engine.offload import OffloadPolicy
from ..logical.assignments import ExternalBlockAssignments
from ..logical.manager import ImmutableBlock, MutableBlock, Tier
from ..logical.sequence import TokenBlockSequence
from ..utils.metrics import CacheStatsTracker
from ..utils.tracing import audit
from .engine import WorkerTierEngine
from .protocol import (ConnectorMetadata, FetchOp, OffloadOp, OnboardOp, PullOp, PushOp, RecvOp, SpillOp, StageOp,
                       StoreOp)

# kv_transfer_params key a decode instance puts on the requests it sends to a prefill instance
REMOTE_DECODE_KEY = "kvbm_remote_decode"


@dataclass
class KvbmRequest:
    request_id: str
    tokens: list[int]
    lora_name: str | None = None
    salt: str | None = None
    max_tokens: int | None = None
    kv_transfer_params: dict | None = None


@dataclass
class RemotePrefill:
    """Decode side: a request whose prefill runs on a prefill instance."""

    params: RemotePrefillParams
    target: int
    slot: int
    seq: int = 0
    provided_blocks: int = 0
    dispatched: bool = False


@dataclass
class PushState:
    """Prefill side: where a remote request's blocks go and how far they went."""

    peer: int
    dst_ids: list[int]        # decode G1 blocks of blocks [provided_blocks, prompt_blocks)
    provided_blocks: int
    slot: int
    seq: int
    cursor: int               # next block index to push
    in_flight: bool = False   # the final push was issued and has not been reported done
    peer_tp: int = 1          # the decode instance's TP degree


@dataclass
class RequestSlot:
    request: KvbmRequest
    seq: TokenBlockSequence
    # the request's G1 block ids, paired with sequence hashes as blocks complete (assigned)
    g1: ExternalBlockAssignments = field(default_factory=ExternalBlockAssignments)
    num_computed_tokens: int = 0
    matched: list[ImmutableBlock] = field(default_factory=list)
    matched_start_block: int = 0
    onboarding: list[ImmutableBlock] = field(default_factory=list)
    save_cursor: int = 0                      # blocks already offloaded (or skipped)
    pending_offload_steps: set[int] = field(default_factory=set)
    finished: bool = False
    remote_future: object = None              # in-flight remote search + pull (concurrent.futures.Future)
    remote_done: bool = False
    cd_decided: bool = False
    remote_prefill: RemotePrefill | None = None
    push: PushState | None = None
    # G3 hits being staged into G2 for this request's onboard: (G3 refs, G2 destinations, hashes)
    staging: tuple[list[ImmutableBlock], list[MutableBlock], list[int]] | None = None
    onboard_pending: bool = False             # an onboard (or stage) was queued and not reported received

    @property
    def g1_block_ids(self) -> list[int]:
        return self.g1.block_ids()


@dataclass
class SchedulerOutputLite:
    """What the connector needs from a scheduler step (framework-agnostic)."""

    step: int
    # req_id -> (new token ids appended, new G1 block ids appended, num_computed_tokens after this step)
    scheduled: dict[str, tuple[list[int], list[int], int]] = field(default_factory=dict)
    finished_req_ids: list[str] = field(default_factory=list)
    # requests the scheduler preempted this step: their G1 blocks return to the framework
    preempted_req_ids: list[str] = field(default_factory=list)


class ConnectorLeader:
    """Scheduler-side connector.

    ``cd`` / ``plane`` / ``prefill_target`` turn on conditional
    disaggregation on a decode instance: ``cd`` decides per request,
    ``plane`` (``engine.cd_plane.PrefillPlane``) carries the dispatch to the
    prefill instance ``prefill_target`` (an instance id, or a callable
    returning one per request), ``mailbox_slots`` bounds the remote prefills
    in flight (one completion word each). Any instance accepts remote
    prefills: a request whose ``kv_transfer_params`` carry
    ``REMOTE_DECODE_KEY`` is pushed to the decode instance named there.
    """

    def __init__(self, leader: InstanceLeader, block_size: int, offload_enabled: bool = True,
                 decode_offload: bool = False, stats: CacheStatsTracker | None = None, remote_search=None,
                 cd: ConditionalDisagg | None = None, plane=None, prefill_target=None, instance_id: int = 0,
                 mailbox_slots: int = 0, recv_timeout_s: float = 120.0, num_workers: int = 1,
                 g2_policy: OffloadPolicy | None = None, g3_policy: OffloadPolicy | None = None,
                 tp_size: int = 1, directory=None, objects=None):
        self.leader = leader
        self.remote = remote_search  # engine.remote_search.RemoteSearch, or None
        self.block_size = block_size
        self.offload_enabled = offload_enabled
        self.decode_offload = decode_offload
        self.slots: dict[str, RequestSlot] = {}
        self.iteration = 0
        self._onboard_ops: list[OnboardOp] = []
        self._recv_ops: list[RecvOp] = []
        self._lock = threading.Lock()
        self.stats = stats or CacheStatsTracker()
        self.cd, self.plane, self.prefill_target = cd, plane, prefill_target
        self.instance_id = instance_id
        self.recv_timeout_s = recv_timeout_s
        self._mailbox_free = deque(range(mailbox_slots))
        self._seq = itertools.count(1)
        self.num_workers = num_workers
        self.tp_size = tp_size          # this instance's TP degree (decode side: its ranks' head shards)
        self.directory = directory      # where prefill instances publish their TP degree
        # the tier engine behind the LeaderEngine seam: G2/G3 state driven by the workers' reports
        self.engine = WorkerTierEngine(leader, num_workers=num_workers, g2_policy=g2_policy, g3_policy=g3_policy,
                                       objects=objects)
        self._fetch_ops: list[FetchOp] = []
        # remote-search pulls the workers run (queued from the remote-search thread, emitted per step)
        self._pull_ops: list[PullOp] = []
        self._pulls: dict[int, list] = {}   # pull id -> [done event, workers reported]
        self._pull_ids = itertools.count(1)
        self._stage_ops: list[StageOp] = []
        self._counts = {"onboarded_blocks": 0, "offload_ops": 0}
        self.cd_stats = {"remote": 0, "local": 0, "dispatched": 0, "received": 0, "failed": 0, "pushed_blocks": 0}

    # ---------------------------------------------------------------- slots
    def create_slot(self, request: KvbmRequest) -> RequestSlot:
        slot = self.slots.get(request.request_id)
        if slot is None:
            salt = request.salt or request.lora_name
            slot = RequestSlot(request, TokenBlockSequence(request.tokens, self.block_size, salt))
            self.slots[request.request_id] = slot
            remote = (request.kv_transfer_params or {}).get(REMOTE_DECODE_KEY)
            if remote is not None:
                # prefill accept: this instance computes the prompt and pushes it to the decode instance
                pb = int(remote["provided_blocks"])
                slot.push = PushState(int(remote["instance"]), list(remote["dst_ids"]), pb, int(remote["slot"]),
                                      int(remote["seq"]), pb, peer_tp=int(remote.get("tp", 1)))
                audit("cd_prefill_accept", request=request.request_id, peer=slot.push.peer,
                      blocks=len(slot.push.dst_ids))
        return slot

    def has_slot(self, req_id: str) -> bool:
        return req_id in self.slots

    # ----------------------------------------------------------------- GNMT
    def get_num_new_matched_tokens(self, req_id: str, num_computed_tokens: int) -> tuple[int | None, bool]:
        slot = self.slots[req_id]
        if slot.remote_prefill is not None:
            return len(slot.request.tokens) - num_computed_tokens, True
        for b in slot.matched:
            b.release()
        slot.matched = []
        hashes = slot.seq.hashes_view()
        start = num_computed_tokens // self.block_size
        if num_computed_tokens % self.block_size or start > len(hashes):
            return 0, False
        blocks: list[ImmutableBlock] = []
        if slot.staging is not None:
            self._release_staging(slot)
        if start < len(hashes):
            blocks = self._find(hashes[start:])
        # the framework must compute at least the last prompt token itself
        max_blocks = (len(slot.request.tokens) - 1 - num_computed_tokens) // self.block_size
        if self.remote is not None and not slot.remote_done and len(blocks) < max_blocks:
            # stall the request while another instance's copy of the missing prefix is pulled
            fut = slot.remote_future
            if fut is None:
                slot.remote_future = self.remote.start(hashes[start + len(blocks): start + max_blocks])
            if not slot.remote_future.done():
                for b in blocks:
                    b.release()
                audit("gnmt_pending", request=req_id)
                return None, False
            slot.remote_done = True
            try:
                pulled = slot.remote_future.result()
            except Exception as e:  # noqa: BLE001 - a failed pull falls back to recompute
                audit("remote_pull_failed", request=req_id, error=str(e))
                pulled = 0
            if pulled:
                for b in blocks:
                    b.release()
                blocks = self._find(hashes[start:])
        for b in blocks[max(0, max_blocks):]:
            b.release()
        blocks = blocks[: max(0, max_blocks)]
        blocks = self._prepare_staging(slot, blocks)
        self.stats.record("host", len(hashes) - start, len(blocks), self.block_size)
        slot.matched = blocks
        slot.matched_start_block = start
        local_tokens = len(blocks) * self.block_size
        if self._decide_remote(slot, num_computed_tokens, local_tokens):
            # the held G2 prefix plus everything the prefill instance computes arrive asynchronously
            return len(slot.request.tokens) - num_computed_tokens, True
        if not blocks:
            return 0, False
        if slot.remote_done:
            audit("gnmt_matched", request=req_id, matched_tokens=local_tokens)
        return local_tokens, True

    @property
    def tier_stats(self) -> dict:
        """Blocks onboarded, offload ops issued, G3 blocks staged into G2 and G2 blocks spilled to G3."""
        e = self.engine.stats
        return {**self._counts, "staged_from_g3": e["staged_from_g3"], "spilled_to_g3": e["spilled_to_g3"]}

    def _find(self, hashes: list[int]) -> list[ImmutableBlock]:
        """G2 prefix, continued in G3 (held, not staged: the workers stage them with the onboard)."""
        return self.engine.match(hashes)

    def _prepare_staging(self, slot: RequestSlot, blocks: list[ImmutableBlock]) -> list[ImmutableBlock]:
        """Give every G3 block of the match a G2 destination; without room in G2 the match stops before G3."""
        blocks, slot.staging = self.engine.prepare_staging(blocks)
        return blocks

    def _release_staging(self, slot: RequestSlot) -> None:
        staging, slot.staging = slot.staging, None
        self.engine.release_staging(staging)

    def _decide_remote(self, slot: RequestSlot, computed: int, local_tokens: int) -> bool:
        """Decode-side CD decision (policy, breaker tier, in-flight budget, a free mailbox slot)."""
        if self.cd is None or self.plane is None or slot.push is not None or slot.cd_decided:
            return False
        slot.cd_decided = True
        total = len(slot.request.tokens)
        if self.cd.decide(total, computed, local_tokens) != Decision.REMOTE:
            self.cd_stats["local"] += 1
            return False
        if not self._mailbox_free:
            self.cd.finish_remote()  # no completion word free: prefill locally
            self.cd_stats["local"] += 1
            return False
        target = self.prefill_target(slot.request) if callable(self.prefill_target) else self.prefill_target
        params = RemotePrefillParams(initiator_instance_id=str(self.instance_id),
                                     decode_endpoint=str(self.instance_id))
        slot.remote_prefill = RemotePrefill(params, int(target), self._mailbox_free.popleft())
        self.cd_stats["remote"] += 1
        audit("cd_decision", request=slot.request.request_id, decision="remote", target=int(target))
        return True

    # ----------------------------------------------------------------- USAA
    def update_state_after_alloc(self, req_id: str, block_ids: list[int], num_external_tokens: int) -> None:
        slot = self.slots[req_id]
        slot.g1.clear()
        slot.g1.extend_block_ids(block_ids)
        if num_external_tokens <= 0:
            for b in slot.matched:
                b.release()
            slot.matched = []
            return
        bs = self.block_size
        start = slot.matched_start_block
        if slot.remote_prefill is not None:
            take = slot.matched
        else:
            n = num_external_tokens // bs
            take, rest = slot.matched[:n], slot.matched[n:]
            for b in rest:
                b.release()
        n = len(take)
        g1 = slot.g1_block_ids[start: start + n]
        if len(g1) != n:
            raise ValueError(f"{req_id}: {n} onboard blocks but only {len(g1)} G1 destinations")
        src_ids = [b.block_id for b in take if b.tier == Tier.G2]
        if slot.staging is not None:
            g3, dst, hashes = slot.staging
            k = n - len(src_ids)  # G3 blocks actually onboarded
            for b in g3[k:]:
                b.release()
            for m in dst[k:]:
                m.release()
            slot.staging = (g3[:k], dst[:k], hashes[:k]) if k else None
            if k:
                # G3 continuations are staged, G4 continuations fetched, into their G2 destinations
                from_disk = [(b, m) for b, m in zip(g3[:k], dst[:k]) if b.tier == Tier.G3]
                from_store = [(b, m) for b, m in zip(g3[:k], dst[:k]) if b.tier == Tier.G4]
                if from_disk:
                    self._stage_ops.append(StageOp(req_id, [b.block_id for b, _ in from_disk],
                                                   [m.block_id for _, m in from_disk]))
                if from_store:
                    self._fetch_ops.append(FetchOp(req_id, [b.sequence_hash for b, _ in from_store],
                                                   [m.block_id for _, m in from_store]))
                src_ids += [m.block_id for m in dst[:k]]
            take = [b for b in take if b.tier == Tier.G2]
        if n:
            self._onboard_ops.append(OnboardOp(req_id, src_ids, g1))
            self._counts["onboarded_blocks"] += n
            slot.onboard_pending = True
        slot.onboarding = take
        slot.matched = []
        # onboarded blocks are already in G2: the save cursor skips past them
        slot.save_cursor = max(slot.save_cursor, start + n)
        if slot.remote_prefill is not None:
            self._dispatch_remote(slot, start + n)

    def _dispatch_remote(self, slot: RequestSlot, provided_blocks: int) -> None:
        """Send the request to its prefill instance; the workers watch its mailbox slot."""
        from ..engine.cd_plane import encode_dispatch

        rp = slot.remote_prefill
        req = slot.request
        bs = self.block_size
        prompt_blocks = (len(req.tokens) + bs - 1) // bs
        if len(slot.g1_block_ids) < prompt_blocks:
            raise ValueError(f"{req.request_id}: {len(slot.g1_block_ids)} G1 blocks for a {prompt_blocks}-block prompt")
        rp.provided_blocks = provided_blocks
        rp.seq = next(self._seq)
        rp.params.num_provided_tokens = provided_blocks * bs
        dst = slot.g1_block_ids[provided_blocks:prompt_blocks]
        decode = {"instance": self.instance_id, "dst_ids": dst, "slot": rp.slot, "seq": rp.seq,
                  "provided_blocks": provided_blocks, "tp": self.tp_size}
        self.plane.dispatch(rp.target, encode_dispatch(req.request_id, slot.seq.tokens, rp.params.to_dict(), decode,
                                                      salt=req.salt, lora=req.lora_name))
        rp.dispatched = True
        self.cd_stats["dispatched"] += 1
        self._recv_ops.append(RecvOp(req.request_id, rp.slot, rp.seq, dst, self.recv_timeout_s,
                                     self._contributors(rp.target)))
        audit("cd_dispatch", request=req.request_id, target=rp.target, provided_blocks=provided_blocks,
              blocks=len(dst), seq=rp.seq)

    def _contributors(self, prefill_instance: int) -> int:
        """Prefill ranks whose pushes fill one of this instance's rank shards."""
        if self.directory is None:
            return 1
        ptp = int(self.directory.lookup(prefill_instance).get("tp", 1))
        return max(1, ptp // self.tp_size)

    # ------------------------------------------------------ metadata build
    def queue_remote_pull(self, pools: list, src_ids: list[int], g2_ids: list[int], timeout: float = 60.0) -> None:
        """Have the workers copy another instance's G2 blocks ``src_ids`` (its pool exports
        ``pools``, one per rank) into this instance's G2 ``g2_ids``; returns once every worker
        reported the copy. Called from a remote-search thread: the op leaves with the next
        step's metadata, so the scheduler must keep stepping meanwhile."""
        ev = threading.Event()
        with self._lock:
            pid = next(self._pull_ids)
            self._pulls[pid] = [ev, 0, False]  # done event, workers reported, a worker failed
            self._pull_ops.append(PullOp(pid, list(pools), [int(i) for i in src_ids], [int(i) for i in g2_ids]))
        try:
            if not ev.wait(timeout):
                raise TimeoutError(f"remote pull {pid}: the workers did not report the copy in {timeout:.0f} s")
            if self._pulls[pid][2]:
                raise RuntimeError(f"remote pull {pid}: a worker could not copy the holder's blocks")
        finally:
            with self._lock:
                self._pulls.pop(pid, None)

    def build_connector_meta(self, out: SchedulerOutputLite) -> bytes:
        self.iteration += 1
        with self._lock:
            pulls, self._pull_ops = self._pull_ops, []
        meta = ConnectorMetadata(step=out.step or self.iteration, onboard=self._onboard_ops, recv=self._recv_ops,
                                 stage=self._stage_ops, pull=pulls, fetch=self._fetch_ops)
        self._onboard_ops, self._recv_ops, self._stage_ops, self._fetch_ops = [], [], [], []
        meta.spill = [SpillOp(g2, g3) for g2, g3 in self.engine.take_spill_ops(meta.step)]
        meta.store = [StoreOp(g2, hs) for g2, hs in self.engine.take_store_ops(meta.step)]
        for req_id in out.preempted_req_ids:
            # The workers fence in-flight offloads of these requests before their G1 blocks are
            # reused (evict list). The request resumes from its token sequence with new G1 blocks;
            # what was saved stays in G2 (present blocks are skipped when it is saved again).
            slot = self.slots.get(req_id)
            if slot is None:
                continue
            meta.evict.append(req_id)
            self.engine.evict(req_id)
            slot.g1.clear()
            slot.save_cursor = 0
            slot.num_computed_tokens = 0
            self.leader.stats["preempted"] = self.leader.stats.get("preempted", 0) + 1
        offloading: dict[str, RequestSlot] = {}
        for req_id, (new_tokens, new_blocks, num_computed) in out.scheduled.items():
            slot = self.slots.get(req_id)
            if slot is None:
                continue
            if new_tokens:
                slot.seq.append(new_tokens)
            if new_blocks:
                slot.g1.extend_block_ids(new_blocks)
            slot.num_computed_tokens = num_computed
            # computed complete blocks take their sequence hashes (assigned, in position order)
            hashes = slot.seq.hashes_view()
            slot.g1.assign_pending(hashes, num_computed // self.block_size)
            if slot.push is not None:
                self._advance_push(slot, num_computed, meta)
            if not self.offload_enabled:
                continue
            complete = slot.g1.assigned_count()
            if not self.decode_offload and num_computed > len(slot.request.tokens):
                complete = min(complete, len(slot.request.tokens) // self.block_size)
            if complete <= slot.save_cursor:
                continue
            self.engine.offload(req_id, hashes[slot.save_cursor: complete],
                                slot.g1.assigned_ids(slot.save_cursor, complete))
            slot.save_cursor = complete
            offloading[req_id] = slot
        # flush: the copies run after this step's forward pass (wait_for_save), never mid-pass
        for req_id, g1_ids, g2_ids in self.engine.take_offload_drain(meta.step):
            meta.offload.append(OffloadOp(req_id, g1_ids, g2_ids))
            offloading[req_id].pending_offload_steps.add(meta.step)
            self.leader.stats["offloaded_blocks"] += len(g1_ids)
            self._counts["offload_ops"] += 1
        return meta.encode()

    def _advance_push(self, slot: RequestSlot, num_computed: int, meta: ConnectorMetadata) -> None:
        """Prefill side: push the blocks whose KV this step computes (the last, partial one with the last chunk)."""
        ps = slot.push
        bs = self.block_size
        prompt_blocks = ps.provided_blocks + len(ps.dst_ids)
        upto = prompt_blocks if num_computed >= len(slot.request.tokens) else num_computed // bs
        upto = min(upto, prompt_blocks, len(slot.g1_block_ids))
        if upto <= ps.cursor:
            return
        src = slot.g1_block_ids[ps.cursor: upto]
        dst = ps.dst_ids[ps.cursor - ps.provided_blocks: upto - ps.provided_blocks]
        final = upto >= prompt_blocks
        meta.push.append(PushOp(slot.request.request_id, ps.peer, src, dst, ps.slot, ps.seq, final, ps.peer_tp))
        ps.cursor = upto
        ps.in_flight = ps.in_flight or final
        self.cd_stats["pushed_blocks"] += len(src)

    # ------------------------------------------------------ worker output
    def update_connector_output(self, finished_sending: set[str] | None = None,
                                finished_recving: set[str] | None = None, worker_meta: dict | None = None,
                                invalid_block_ids: set[int] | None = None) -> None:
        if worker_meta and (worker_meta.get("pulled") or worker_meta.get("pull_failed")):
            worker_meta = dict(worker_meta)
            with self._lock:
                for kind in ("pulled", "pull_failed"):
                    for pid, n in (worker_meta.pop(kind, None) or {}).items():
                        p = self._pulls.get(int(pid))
                        if p is None:
                            continue
                        p[1] += int(n)
                        p[2] = p[2] or kind == "pull_failed"
                        if p[1] >= self.num_workers:
                            p[0].set()
        self.engine.on_worker_report(worker_meta)
        bad = set(invalid_block_ids or ())
        for req_id in finished_recving or ():
            slot = self.slots.get(req_id)
            if slot is None:
                continue
            for b in slot.onboarding:
                b.release()
            slot.onboarding = []
            slot.onboard_pending = False
            if slot.staging is not None:
                # the stage ran before the onboard that finished: the G2 copies hold the data now
                staging, slot.staging = slot.staging, None
                self.engine.finish_staging(staging)
            rp = slot.remote_prefill
            if rp is not None:
                failed = bool(bad.intersection(slot.g1_block_ids))
                self._close_remote(slot, failed)
            if slot.finished and not slot.pending_offload_steps:
                self._drop(req_id)
        for req_id in finished_sending or ():
            slot = self.slots.get(req_id)
            if slot is not None:
                slot.pending_offload_steps.clear()
                if slot.push is not None:
                    slot.push.in_flight = False
                if slot.finished:
                    self._drop(req_id)

    def _close_remote(self, slot: RequestSlot, failed: bool) -> None:
        rp = slot.remote_prefill
        slot.remote_prefill = None
        self._mailbox_free.append(rp.slot)
        if self.cd is not None:
            self.cd.finish_remote()
        self.cd_stats["failed" if failed else "received"] += 1
        audit("cd_received", request=slot.request.request_id, seq=rp.seq, failed=failed)

    def request_finished(self, req_id: str, block_ids: list[int] | None = None) -> tuple[bool, dict | None]:
        slot = self.slots.get(req_id)
        if slot is None:
            return False, None
        slot.finished = True
        if slot.staging is not None and not slot.onboard_pending:
            self._release_staging(slot)
        for b in slot.matched + slot.onboarding:
            b.release()
        slot.matched, slot.onboarding = [], []
        if slot.remote_prefill is not None and slot.remote_prefill.dispatched:
            # finished (e.g. aborted) before its KV arrived: the workers still watch the slot
            return True, None
        if slot.pending_offload_steps or (slot.push is not None and slot.push.in_flight):
            return True, None  # the worker reports it in finished_sending when its copies are done
        self._drop(req_id)
        return False, None

    def _drop(self, req_id: str) -> None:
        self.slots.pop(req_id, None)

    def num_slots(self) -> int:
        return len(self.slots)
