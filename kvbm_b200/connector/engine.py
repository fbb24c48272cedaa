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
from ..logical.manager import ImmutableBlock
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
