"""The seam between a connector and the block-management engine.

A connector (the vLLM hooks, or any other framework's) drives requests
through a :class:`LeaderEngine`; the engine owns searches, onboards and
offloads and hands back ids the connector polls and releases:

* ``find_blocks(req, hashes)`` -> :class:`SearchHandle`: local G2/G3 match,
  then (optionally) a remote search; ``poll_search`` reports PENDING until
  it settles, then the matched G2 blocks (held until ``release_search``).
* ``onboard_blocks(req, search, g1_ids)`` -> action id: copies the search's
  blocks into G1; ``poll_action`` reports PENDING / DONE / FAILED and
  ``release_action`` drops the engine's references.
* ``offload(req, hashes, g1_ids)`` buffers G1 blocks for the G1 -> G2
  pipeline; ``take_offload_drain`` flushes the buffer once the forward pass
  that wrote them has finished (never enqueue a G1 read mid-pass);
  ``evict(req)`` drops a request's pending offloads.
* ``release_prefill_session(session)`` ends a conditional-disaggregation
  prefill session.

:class:`LocalConnectorEngine` implements it over an ``InstanceLeader`` (plus
an optional ``RemoteSearch``); :class:`NoopBlockEngine` finds nothing and
offloads nothing (KVBM disabled).

Parity: crates/kvbm-protocols/src/connector/{engine.rs (LeaderEngine),
handles.rs, noop.rs (NoopBlockEngine)}, crates/kvbm-engine/src/tiering/
engine/{local.rs, find.rs, onboard.rs, offload.rs} (LocalConnectorEngine,
buffer-then-flush offload).
"""

from __future__ import annotations

import enum
import itertools
import threading
from dataclasses import dataclass, field

from ..engine.leader import FindMatchesOptions, InstanceLeader
from ..logical.manager import ImmutableBlock, Tier
from ..utils.tracing import audit


class Status(str, enum.Enum):
    PENDING = "pending"
    READY = "ready"
    DONE = "done"
    FAILED = "failed"
    RELEASED = "released"


@dataclass
class SearchHandle:
    search_id: int
    request_id: str
    status: Status = Status.PENDING
    blocks: list[ImmutableBlock] = field(default_factory=list)
    error: str | None = None

    @property
    def num_blocks(self) -> int:
        return len(self.blocks)


class LeaderEngine:
    def find_blocks(self, request_id: str, hashes: list[int]) -> SearchHandle:
        raise NotImplementedError

    def poll_search(self, search_id: int) -> SearchHandle:
        raise NotImplementedError

    def release_search(self, search_id: int) -> None:
        raise NotImplementedError

    def onboard_blocks(self, request_id: str, search_id: int, g1_ids: list[int]) -> int:
        raise NotImplementedError

    def poll_action(self, action_id: int) -> Status:
        raise NotImplementedError

    def release_action(self, action_id: int) -> None:
        raise NotImplementedError

    def offload(self, request_id: str, hashes: list[int], g1_ids: list[int]) -> None:
        raise NotImplementedError

    def take_offload_drain(self) -> list:
        raise NotImplementedError

    def evict(self, request_id: str) -> int:
        raise NotImplementedError

    def release_prefill_session(self, session_id: str) -> None:
        raise NotImplementedError


class NoopBlockEngine(LeaderEngine):
    """Finds nothing, moves nothing: the engine of a connector with KVBM turned off."""

    def __init__(self):
        self._ids = itertools.count(1)

    def find_blocks(self, request_id, hashes):
        return SearchHandle(next(self._ids), request_id, Status.READY)

    def poll_search(self, search_id):
        return SearchHandle(search_id, "", Status.READY)

    def release_search(self, search_id):
        pass

    def onboard_blocks(self, request_id, search_id, g1_ids):
        if g1_ids:
            raise ValueError("the no-op engine has nothing to onboard")
        return 0

    def poll_action(self, action_id):
        return Status.DONE

    def release_action(self, action_id):
        pass

    def offload(self, request_id, hashes, g1_ids):
        pass

    def take_offload_drain(self):
        return []

    def evict(self, request_id):
        return 0

    def release_prefill_session(self, session_id):
        pass


class LocalConnectorEngine(LeaderEngine):
    """``LeaderEngine`` over this process's ``InstanceLeader`` (and an optional ``RemoteSearch``)."""

    def __init__(self, leader: InstanceLeader, remote_search=None, sessions=None):
        self.leader, self.remote, self.sessions = leader, remote_search, sessions
        self._ids = itertools.count(1)
        self._lock = threading.Lock()
        self._searches: dict[int, tuple[SearchHandle, list[int], object]] = {}
        self._actions: dict[int, tuple[object, list[ImmutableBlock]]] = {}
        self._offload_buf: list[tuple[str, list[int], list[int]]] = []

    # ------------------------------------------------------------ search
    def find_blocks(self, request_id, hashes):
        h = SearchHandle(next(self._ids), request_id)
        res = self.leader.find_matches(list(hashes), FindMatchesOptions())
        fut = None
        if self.remote is not None and len(res.g2_blocks) < len(hashes):
            fut = self.remote.start(list(hashes[len(res.g2_blocks):]))
            h.blocks = res.g2_blocks  # held meanwhile; re-matched when the pull lands
        else:
            h.blocks, h.status = res.g2_blocks, Status.READY
        with self._lock:
            self._searches[h.search_id] = (h, list(hashes), fut)
        audit("find_blocks", request=request_id, search=h.search_id, local=len(res.g2_blocks),
              remote=fut is not None)
        return h

    def poll_search(self, search_id):
        with self._lock:
            h, hashes, fut = self._searches[search_id]
        if h.status != Status.PENDING:
            return h
        if not fut.done():
            return h
        try:
            pulled = fut.result()
        except Exception as e:  # noqa: BLE001 - a failed pull leaves the local match
            h.error, pulled = str(e), 0
        if pulled:
            for b in h.blocks:
                b.release()
            h.blocks = self.leader.find_matches(hashes, FindMatchesOptions()).g2_blocks
        h.status = Status.READY
        return h

    def release_search(self, search_id):
        with self._lock:
            entry = self._searches.pop(search_id, None)
        if entry is not None:
            for b in entry[0].blocks:
                b.release()
            entry[0].blocks, entry[0].status = [], Status.RELEASED

    # ----------------------------------------------------------- onboard
    def onboard_blocks(self, request_id, search_id, g1_ids):
        with self._lock:
            h, _, _ = self._searches[search_id]
        if h.status != Status.READY:
            raise RuntimeError(f"search {search_id} is {h.status.value}")
        n = len(g1_ids)
        if n > len(h.blocks):
            raise ValueError(f"{n} G1 destinations for {len(h.blocks)} matched blocks")
        take, rest = h.blocks[:n], h.blocks[n:]
        for b in rest:
            b.release()
        h.blocks = []
        note = self.leader.onboard(take, list(g1_ids))
        aid = next(self._ids)
        with self._lock:
            self._actions[aid] = (note, take)
        return aid

    def poll_action(self, action_id):
        with self._lock:
            entry = self._actions.get(action_id)
        if entry is None:
            return Status.RELEASED
        note, _ = entry
        try:
            return Status.DONE if (note is None or note.is_complete()) else Status.PENDING
        except Exception:  # noqa: BLE001
            return Status.FAILED

    def release_action(self, action_id):
        with self._lock:
            entry = self._actions.pop(action_id, None)
        if entry is not None:
            note, blocks = entry
            if note is not None:
                note.wait()
            for b in blocks:
                b.release()

    # ----------------------------------------------------------- offload
    def offload(self, request_id, hashes, g1_ids):
        if len(hashes) != len(g1_ids):
            raise ValueError("one G1 block per hash")
        with self._lock:
            self._offload_buf.append((request_id, list(hashes), list(g1_ids)))

    def take_offload_drain(self):
        """Flush the buffered offloads (call after the forward pass that wrote them)."""
        with self._lock:
            buf, self._offload_buf = self._offload_buf, []
        return [(rid, self.leader.offload_g1(hs, ids)) for rid, hs, ids in buf]

    def evict(self, request_id):
        with self._lock:
            before = len(self._offload_buf)
            self._offload_buf = [e for e in self._offload_buf if e[0] != request_id]
            return before - len(self._offload_buf)

    def release_prefill_session(self, session_id):
        if self.sessions is None:
            return
        try:
            s = self.sessions.get(session_id)
        except KeyError:
            return
        s.close("released")
        self.sessions.remove(session_id)


class ObjectHit:
    """A G4 (object store) match: no block pool holds it, so it has no block id and no reference."""

    tier = Tier.G4
    block_id = -1

    def __init__(self, seq_hash: int):
        self.sequence_hash = int(seq_hash)

    def release(self) -> None:
        pass


class WorkerTierEngine(LocalConnectorEngine):
    """``LeaderEngine`` of a connector whose workers live in other processes.

    The leader cannot move bytes itself: every copy becomes an op in the
    step metadata that the workers run (onboard, offload, stage, spill), and
    the tier state follows the workers' reports:

    * :meth:`match` - G2 prefix continued in G3; G3 hits are held, not
      staged (``StagingMode.PREPARE``);
    * :meth:`prepare_staging` / :meth:`finish_staging` - G2 destinations for
      held G3 hits, registered in G2 once the onboard that follows the stage
      is reported received;
    * :meth:`offload` (buffer) / :meth:`take_offload_drain` (flush, once per
      step, after the pass that wrote the blocks): the G1 -> G2 policy,
      skipping hashes G2 holds or has in flight, G2 destinations allocated
      (evicting inactive blocks), returned as offload ops;
    * :meth:`on_worker_report` - G2 destinations registered when every
      worker reported the step's copies; registered G2 blocks pass the G3
      policy and are queued as spill ops (:meth:`take_spill_ops`), the G3
      copies registered when the spill is reported.

    With an object store (``objects``): the match continues past G2 / G3 into
    G4 (every rank's object present), G4 hits get G2 destinations like G3
    hits and are fetched by the workers before the onboard (fetch ops);
    registered G2 blocks the store does not hold yet are uploaded by the
    workers (store ops), their G2 references held until every worker
    reported the upload.

    Parity: crates/kvbm-engine/src/tiering/engine/{local.rs, find.rs,
    offload.rs} (buffer, flush at finish_forward_pass), tiering/offload/
    engine.rs:123 (register after the transfer), the G2 -> G3 auto-chain,
    the G2 -> G4 chain with its object-presence policy, remote/search/g4.rs.
    """

    def __init__(self, leader: InstanceLeader, num_workers: int = 1, g2_policy=None, g3_policy=None,
                 remote_search=None, sessions=None, objects=None):
        from ..engine.offload import PresenceFilter

        super().__init__(leader, remote_search, sessions)
        self.num_workers = num_workers
        self.g2_policy = g2_policy or PresenceFilter(leader.g2)
        self.g3_policy = g3_policy or (PresenceFilter(leader.g3) if leader.g3 is not None else None)
        self._buffer: list[tuple[str, list[int], list[int]]] = []
        # step -> (G2 mutables awaiting their copies, their hashes, worker reports so far)
        self._pending_g2: dict[int, tuple[list[int], list[int], int]] = {}  # bare G2 ids owned until registered
        self._spill_queue: list[tuple[list[ImmutableBlock], list, list[int]]] = []
        # step -> (G3 mutables awaiting the spill copies, hashes, G2 sources held, worker reports so far)
        self._pending_g3: dict[int, tuple[list, list[int], list[ImmutableBlock], int]] = {}
        # G4: the store (presence checks here; the workers move the bytes), uploads queued / in flight
        self.objects = objects
        self._store_queue: list[tuple[list[ImmutableBlock], list[int]]] = []
        self._pending_g4: dict[int, tuple[list[ImmutableBlock], list[int], int]] = {}
        self.stats = {"offloaded_blocks": 0, "staged_from_g3": 0, "spilled_to_g3": 0, "offload_ops": 0,
                      "staged_from_g4": 0, "stored_to_g4": 0}

    def _in_store(self, seq_hash: int) -> bool:
        return all(self.objects.has(self.objects.key(seq_hash, rank=r)) for r in range(self.num_workers))

    # ------------------------------------------------------------- find
    def match(self, hashes: list[int]) -> list[ImmutableBlock]:
        from ..engine.leader import StagingMode

        res = self.leader.find_matches(list(hashes), FindMatchesOptions(staging=StagingMode.PREPARE))
        out = res.g2_blocks + res.g3_held
        if self.objects is not None:
            for h in list(hashes)[len(out):]:  # the prefix continues in the object store
                if not self._in_store(h):
                    break
                out.append(ObjectHit(h))
        return out

    def prepare_staging(self, blocks: list[ImmutableBlock]):
        """(blocks the onboard can use, staging) - G3 hits get G2 destinations; without room in G2 the
        match stops before G3. ``staging`` is (G3 refs, G2 destinations, hashes) or None."""
        from ..logical.manager import Tier

        g3 = [b for b in blocks if b.tier != Tier.G2]  # G3 blocks, then G4 hits
        if not g3:
            return blocks, None
        got = self.leader.g2.allocate_blocks_with_evictions(len(g3))
        if got is None:
            for b in g3:
                b.release()
            return blocks[: len(blocks) - len(g3)], None
        return blocks, (g3, got[0], [b.sequence_hash for b in g3])

    @staticmethod
    def release_staging(staging) -> None:
        g3, dst, _ = staging
        for b in g3:
            b.release()
        for m in dst:
            m.release()

    def finish_staging(self, staging) -> None:
        """The stage / fetch ran before the onboard that was reported: the G2 copies hold the data now."""
        g3, dst, hashes = staging
        for b in self.leader.g2.register_mutable(dst, hashes):
            b.release()
        for b in g3:
            b.release()
        n4 = sum(1 for b in g3 if b.tier == Tier.G4)
        self.stats["staged_from_g3"] += len(dst) - n4
        self.stats["staged_from_g4"] += n4

    # ---------------------------------------------------------- offload
    def offload(self, request_id, hashes, g1_ids):
        if len(hashes) != len(g1_ids):
            raise ValueError("one G1 block per hash")
        self._buffer.append((request_id, list(hashes), list(g1_ids)))

    def evict(self, request_id):
        before = len(self._buffer)
        self._buffer = [e for e in self._buffer if e[0] != request_id]
        return before - len(self._buffer)

    def take_offload_drain(self, step: int = 0) -> list:
        """Flush the buffered offloads into this step's ops: ``[(request_id, g1_ids, g2_ids)]``."""
        from ..engine.offload import OffloadItem

        buf, self._buffer = self._buffer, []
        g2 = self.leader.g2
        reg, tier = g2.registry, int(g2.tier)
        pending = self._pending_hashes()
        ops, dsts, hashes_all = [], [], []
        for rid, hashes, g1_ids in buf:
            todo = [(h, b) for h, b in zip(hashes, g1_ids)
                    if h not in pending and self.g2_policy.keep(OffloadItem(h, b)) and not reg.is_present(h, tier)]
            if not todo:
                continue
            dst = g2.allocate_ids_with_evictions(len(todo))  # bare ids: registered or released below
            if dst is None:
                continue  # G2 full of active blocks: skip this offload
            pending |= {h for h, _ in todo}
            ops.append((rid, [b for _, b in todo], dst))
            dsts.extend(dst)
            hashes_all.extend(h for h, _ in todo)
            self.stats["offloaded_blocks"] += len(todo)
            self.stats["offload_ops"] += 1
        if dsts:
            # registered (and so matchable) only once every worker reports these copies done
            self._pending_g2[step] = (dsts, hashes_all, 0)
        return ops

    def _pending_hashes(self) -> set[int]:
        return {h for _, hs, _ in self._pending_g2.values() for h in hs}

    def take_spill_ops(self, step: int) -> list[tuple[list[int], list[int]]]:
        """G2 -> G3 copies for this step's metadata: ``[(g2_ids, g3_ids)]``."""
        if not self._spill_queue:
            return []
        ops, srcs, dsts, hs = [], [], [], []
        for g2_refs, g3_dst, hashes in self._spill_queue:
            ops.append(([b.block_id for b in g2_refs], [m.block_id for m in g3_dst]))
            srcs += g2_refs
            dsts += g3_dst
            hs += hashes
        self._spill_queue = []
        self._pending_g3[step] = (dsts, hs, srcs, 0)
        return ops

    def take_store_ops(self, step: int) -> list[tuple[list[int], list[int]]]:
        """G2 -> G4 uploads for this step's metadata: ``[(g2_ids, hashes)]``."""
        if not self._store_queue:
            return []
        ops, refs, hs = [], [], []
        for g2_refs, hashes in self._store_queue:
            ops.append(([b.block_id for b in g2_refs], list(hashes)))
            refs += g2_refs
            hs += hashes
        self._store_queue = []
        self._pending_g4[step] = (refs, hs, 0)
        return ops

    def _chain_to_g4(self, imm: list[ImmutableBlock]) -> None:
        if self.objects is None or not imm:
            return
        pending = {h for _, hs, _ in self._pending_g4.values() for h in hs}
        pending |= {h for _, hs in self._store_queue for h in hs}
        keep = [b for b in imm if b.sequence_hash not in pending and not self._in_store(b.sequence_hash)]
        if keep:
            self._store_queue.append(([b.clone() for b in keep], [b.sequence_hash for b in keep]))

    def _register_stored(self, stored: dict) -> None:
        for step, n in stored.items():
            step = int(step)
            entry = self._pending_g4.get(step)
            if entry is None:
                continue
            refs, hashes, seen = entry
            seen += int(n)
            if seen < self.num_workers:
                self._pending_g4[step] = (refs, hashes, seen)
                continue
            del self._pending_g4[step]
            for b in refs:
                b.release()
            self.stats["stored_to_g4"] += len(hashes)

    # --------------------------------------------------- worker reports
    def on_worker_report(self, meta: dict | None) -> None:
        if not meta:
            return
        self._register_landed(meta.get("offloaded", {}))
        self._register_spilled(meta.get("spilled", {}))
        self._register_stored(meta.get("stored", {}))

    def _register_landed(self, offloaded: dict) -> None:
        for step, n in offloaded.items():
            step = int(step)
            entry = self._pending_g2.get(step)
            if entry is None:
                continue
            blocks, hashes, seen = entry
            seen += int(n)
            if seen < self.num_workers:
                self._pending_g2[step] = (blocks, hashes, seen)
                continue
            del self._pending_g2[step]
            if self.leader.g3 is None and self.objects is None:
                self.leader.g2.register_ids_released(blocks, hashes)  # cached in G2 (inactive, matchable)
                continue
            imm = self.leader.g2.register_ids(blocks, hashes)
            self._chain_to_g3(imm)
            self._chain_to_g4(imm)
            for b in imm:
                b.release()  # cached in G2 (inactive, matchable)

    def _chain_to_g3(self, imm: list[ImmutableBlock]) -> None:
        from ..engine.offload import OffloadItem

        g3 = self.leader.g3
        if g3 is None or not imm:
            return
        pending = {h for _, hs, _, _ in self._pending_g3.values() for h in hs}
        pending |= {h for _, _, hs in self._spill_queue for h in hs}
        keep = [b for b in imm if b.sequence_hash not in pending
                and self.g3_policy.keep(OffloadItem(b.sequence_hash, b.block_id))]
        if not keep:
            return
        got = g3.allocate_blocks_with_evictions(len(keep))
        if got is None:
            return
        self._spill_queue.append(([b.clone() for b in keep], got[0], [b.sequence_hash for b in keep]))

    def _register_spilled(self, spilled: dict) -> None:
        for step, n in spilled.items():
            step = int(step)
            entry = self._pending_g3.get(step)
            if entry is None:
                continue
            dst, hashes, srcs, seen = entry
            seen += int(n)
            if seen < self.num_workers:
                self._pending_g3[step] = (dst, hashes, srcs, seen)
                continue
            del self._pending_g3[step]
            for b in self.leader.g3.register_mutable(dst, hashes):
                b.release()
            for b in srcs:
                b.release()
            self.stats["spilled_to_g3"] += len(dst)
