"""Scheduler-side connector: per-request slots over the InstanceLeader.

Hooks (called by the serving framework's scheduler, one process):

* ``get_num_new_matched_tokens(req_id, num_computed_tokens)`` - how many
  tokens beyond the framework's own G1 prefix hit can be loaded from G2/G3;
  matched G2 blocks are held by the slot;
* ``update_state_after_alloc(req_id, block_ids, num_external_tokens)`` -
  records the G1 destinations and queues the G2 -> G1 onboard;
* ``build_connector_meta(scheduler_output)`` - advances every scheduled
  request's save cursor: blocks that became complete this step get G2 slots
  (skipping hashes G2 already holds), are registered in G2 and queued as
  G1 -> G2 offloads; returns the step's serialized ops for the workers;
* ``update_connector_output(finished_sending, finished_recving)`` - releases
  onboarded G2 references and acknowledges finished offloads;
* ``request_finished(req_id)`` - asks the framework to delay freeing G1
  blocks while an offload still reads them.

Parity: crates/kvbm-connector/src/connector/leader/mod.rs:139-723 (Leader:
gnmt :449, usaa :462, build_connector_meta :493, request_finished :570,
update_connector_output :559), python/kvbm/vllm/connector/leader.py:50-347.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field

from ..engine.leader import FindMatchesOptions, InstanceLeader
from ..logical.manager import ImmutableBlock
from ..logical.sequence import TokenBlockSequence
from ..utils.metrics import CacheStatsTracker
from ..utils.tracing import audit
from .protocol import ConnectorMetadata, OffloadOp, OnboardOp


@dataclass
class KvbmRequest:
    request_id: str
    tokens: list[int]
    lora_name: str | None = None
    salt: str | None = None
    max_tokens: int | None = None
    kv_transfer_params: dict | None = None


@dataclass
class RequestSlot:
    request: KvbmRequest
    seq: TokenBlockSequence
    g1_block_ids: list[int] = field(default_factory=list)
    num_computed_tokens: int = 0
    matched: list[ImmutableBlock] = field(default_factory=list)
    matched_start_block: int = 0
    onboarding: list[ImmutableBlock] = field(default_factory=list)
    save_cursor: int = 0                      # blocks already offloaded (or skipped)
    pending_offload_steps: set[int] = field(default_factory=set)
    finished: bool = False
    remote_future: object = None              # in-flight remote search + pull (concurrent.futures.Future)
    remote_done: bool = False


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
    def __init__(self, leader: InstanceLeader, block_size: int, offload_enabled: bool = True,
                 decode_offload: bool = False, stats: CacheStatsTracker | None = None, remote_search=None):
        self.leader = leader
        self.remote = remote_search  # engine.remote_search.RemoteSearch, or None
        self.block_size = block_size
        self.offload_enabled = offload_enabled
        self.decode_offload = decode_offload
        self.slots: dict[str, RequestSlot] = {}
        self.iteration = 0
        self._onboard_ops: list[OnboardOp] = []
        self._lock = threading.Lock()
        self.stats = stats or CacheStatsTracker()

    # ---------------------------------------------------------------- slots
    def create_slot(self, request: KvbmRequest) -> RequestSlot:
        slot = self.slots.get(request.request_id)
        if slot is None:
            salt = request.salt or request.lora_name
            slot = RequestSlot(request, TokenBlockSequence(request.tokens, self.block_size, salt))
            self.slots[request.request_id] = slot
        return slot

    def has_slot(self, req_id: str) -> bool:
        return req_id in self.slots

    # ----------------------------------------------------------------- GNMT
    def get_num_new_matched_tokens(self, req_id: str, num_computed_tokens: int) -> tuple[int | None, bool]:
        slot = self.slots[req_id]
        for b in slot.matched:
            b.release()
        slot.matched = []
        hashes = slot.seq.sequence_hashes
        start = num_computed_tokens // self.block_size
        if num_computed_tokens % self.block_size or start >= len(hashes):
            return 0, False
        res = self.leader.find_matches(hashes[start:], FindMatchesOptions())
        blocks = res.g2_blocks
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
                blocks = self.leader.find_matches(hashes[start:], FindMatchesOptions()).g2_blocks
        for b in blocks[max(0, max_blocks):]:
            b.release()
        blocks = blocks[: max(0, max_blocks)]
        self.stats.record("host", len(hashes) - start, len(blocks), self.block_size)
        if not blocks:
            return 0, False
        slot.matched = blocks
        slot.matched_start_block = start
        if slot.remote_done:
            audit("gnmt_matched", request=req_id, matched_tokens=len(blocks) * self.block_size)
        return len(blocks) * self.block_size, True

    # ----------------------------------------------------------------- USAA
    def update_state_after_alloc(self, req_id: str, block_ids: list[int], num_external_tokens: int) -> None:
        slot = self.slots[req_id]
        slot.g1_block_ids = list(block_ids)
        if num_external_tokens <= 0:
            for b in slot.matched:
                b.release()
            slot.matched = []
            return
        n = num_external_tokens // self.block_size
        take, rest = slot.matched[:n], slot.matched[n:]
        for b in rest:
            b.release()
        start = slot.matched_start_block
        g1 = slot.g1_block_ids[start: start + n]
        if len(g1) != n:
            raise ValueError(f"{req_id}: {n} onboard blocks but only {len(g1)} G1 destinations")
        self._onboard_ops.append(OnboardOp(req_id, [b.block_id for b in take], g1))
        slot.onboarding = take
        slot.matched = []
        # onboarded blocks are already in G2: the save cursor skips past them
        slot.save_cursor = max(slot.save_cursor, start + n)

    # ------------------------------------------------------ metadata build
    def build_connector_meta(self, out: SchedulerOutputLite) -> bytes:
        self.iteration += 1
        meta = ConnectorMetadata(step=out.step or self.iteration, onboard=self._onboard_ops)
        self._onboard_ops = []
        for req_id in out.preempted_req_ids:
            # The workers fence in-flight offloads of these requests before their G1 blocks are
            # reused (evict list). The request resumes from its token sequence with new G1 blocks;
            # what was saved stays in G2 (present blocks are skipped when it is saved again).
            slot = self.slots.get(req_id)
            if slot is None:
                continue
            meta.evict.append(req_id)
            slot.g1_block_ids = []
            slot.save_cursor = 0
            slot.num_computed_tokens = 0
            self.leader.stats["preempted"] = self.leader.stats.get("preempted", 0) + 1
        for req_id, (new_tokens, new_blocks, num_computed) in out.scheduled.items():
            slot = self.slots.get(req_id)
            if slot is None:
                continue
            if new_tokens:
                slot.seq.append(new_tokens)
            slot.g1_block_ids.extend(new_blocks)
            slot.num_computed_tokens = num_computed
            if not self.offload_enabled:
                continue
            complete = min(num_computed // self.block_size, slot.seq.num_complete_blocks, len(slot.g1_block_ids))
            if not self.decode_offload and num_computed > len(slot.request.tokens):
                complete = min(complete, len(slot.request.tokens) // self.block_size)
            if complete <= slot.save_cursor:
                continue
            hashes = slot.seq.sequence_hashes[slot.save_cursor: complete]
            g1 = slot.g1_block_ids[slot.save_cursor: complete]
            reg = self.leader.g2.registry
            tier = int(self.leader.g2.tier)
            todo = [(h, b) for h, b in zip(hashes, g1) if not reg.is_present(h, tier)]
            slot.save_cursor = complete
            if not todo:
                continue
            got = self.leader.g2.allocate_blocks_with_evictions(len(todo))
            if got is None:
                continue  # G2 full of active blocks: skip this offload
            dst, _ = got
            imm = self.leader.g2.register_mutable(dst, [h for h, _ in todo])
            meta.offload.append(OffloadOp(req_id, [b for _, b in todo], [d.block_id for d in imm]))
            slot.pending_offload_steps.add(meta.step)
            for b in imm:
                b.release()  # cached in G2 (inactive) once the worker's copy lands
            self.leader.stats["offloaded_blocks"] += len(todo)
        return meta.encode()

    # ------------------------------------------------------ worker output
    def update_connector_output(self, finished_sending: set[str] | None = None,
                                finished_recving: set[str] | None = None) -> None:
        for req_id in finished_recving or ():
            slot = self.slots.get(req_id)
            if slot is not None:
                for b in slot.onboarding:
                    b.release()
                slot.onboarding = []
        for req_id in finished_sending or ():
            slot = self.slots.get(req_id)
            if slot is not None:
                slot.pending_offload_steps.clear()
                if slot.finished:
                    self._drop(req_id)

    def request_finished(self, req_id: str, block_ids: list[int] | None = None) -> tuple[bool, dict | None]:
        slot = self.slots.get(req_id)
        if slot is None:
            return False, None
        slot.finished = True
        for b in slot.matched + slot.onboarding:
            b.release()
        slot.matched, slot.onboarding = [], []
        if slot.pending_offload_steps:
            return True, None  # the worker reports it in finished_sending when its copies are done
        self._drop(req_id)
        return False, None

    def _drop(self, req_id: str) -> None:
        self.slots.pop(req_id, None)

    def num_slots(self) -> int:
        return len(self.slots)
