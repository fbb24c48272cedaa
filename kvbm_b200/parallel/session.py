"""P2P transfer sessions: a per-request stream of commitments and
availability between two instances.

The *initiator* (decode side) opens a session with the *holder* (prefill
side, or a peer holding a cached prefix). The holder announces blocks it
**commits** to provide (by sequence hash) and later marks them **available**
once their KV is in place; the puller drains availability and pulls (or, on
one NVLink box, the holder pushes with the fused kernel and availability
means "already written"). Invariants enforced here:

* available is a subset of committed, both grow monotonically;
* ``finish_commits`` / ``finish_availability`` close the streams;
* a session that is not attached within ``attach_timeout`` is evicted by
  the :class:`SessionManager` watchdog, and ``close(reason)`` fails it with a
  lifecycle event the other side observes.

Parity: crates/kvbm-engine/src/p2p/session/{mod.rs:4-312 (Session trait and
invariants), manager.rs:28-44 (watchdog), testing.rs (MockSession),
velo.rs (wire frames Attach/Commit/CommitsClosed/Available/Drained/Finished),
CONTRACT.md}.
"""

from __future__ import annotations

import enum
import threading
import time
import uuid
from dataclasses import dataclass, field

from ..utils.tracing import audit


class Lifecycle(str, enum.Enum):
    OPEN = "open"
    ATTACHED = "attached"
    COMMITS_CLOSED = "commits_closed"
    DRAINED = "drained"
    FINISHED = "finished"
    FAILED = "failed"


class SessionError(RuntimeError):
    pass


@dataclass
class Session:
    session_id: str = field(default_factory=lambda: uuid.uuid4().hex)
    initiator: int = 0
    holder: int = 0
    created: float = field(default_factory=time.monotonic)

    def __post_init__(self):
        self._cv = threading.Condition()
        self._committed: list[int] = []
        self._committed_set: set[int] = set()
        self._available: list[int] = []
        self._available_set: set[int] = set()
        self._commits_closed = False
        self._avail_closed = False
        self.lifecycle = Lifecycle.OPEN
        self.failure: str | None = None
        self.attached = False
        self._cursor = 0

    # --------------------------------------------------------- holder side
    def attach(self) -> None:
        with self._cv:
            self._check()
            self.attached = True
            if self.lifecycle == Lifecycle.OPEN:
                self.lifecycle = Lifecycle.ATTACHED
            self._cv.notify_all()

    def commit(self, hashes: list[int]) -> None:
        with self._cv:
            self._check()
            if self._commits_closed:
                raise SessionError("commits already closed")
            for h in hashes:
                if h not in self._committed_set:
                    self._committed_set.add(h)
                    self._committed.append(h)
            self._cv.notify_all()

    def finish_commits(self) -> None:
        with self._cv:
            self._commits_closed = True
            if self.lifecycle in (Lifecycle.OPEN, Lifecycle.ATTACHED):
                self.lifecycle = Lifecycle.COMMITS_CLOSED
            self._cv.notify_all()

    def make_available(self, hashes: list[int]) -> None:
        with self._cv:
            self._check()
            missing = [h for h in hashes if h not in self._committed_set]
            if missing:
                raise SessionError(f"{len(missing)} blocks made available without a commitment")
            for h in hashes:
                if h not in self._available_set:
                    self._available_set.add(h)
                    self._available.append(h)
            self._cv.notify_all()

    def finish_availability(self) -> None:
        with self._cv:
            if not self._commits_closed:
                raise SessionError("close commits before availability")
            if self._available_set != self._committed_set:
                raise SessionError("availability closed before every commitment was made available")
            self._avail_closed = True
            self.lifecycle = Lifecycle.DRAINED
            self._cv.notify_all()

    # ------------------------------------------------------- initiator side
    def commits(self) -> list[int]:
        with self._cv:
            return list(self._committed)

    def availability(self) -> list[int]:
        with self._cv:
            return list(self._available)

    def drain_available(self, timeout: float | None = None) -> list[int]:
        """New available hashes since the last call (blocks until some arrive or the stream ends)."""
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._cv:
            while self._cursor >= len(self._available) and not self._avail_closed:
                self._check()
                rem = None if deadline is None else deadline - time.monotonic()
                if rem is not None and rem <= 0:
                    raise TimeoutError("no availability within the timeout")
                self._cv.wait(rem)
            self._check()
            out = self._available[self._cursor:]
            self._cursor = len(self._available)
            return out

    def wait_attached(self, timeout: float) -> None:
        with self._cv:
            ok = self._cv.wait_for(lambda: self.attached or self.failure, timeout)
            self._check()
            if not ok:
                raise TimeoutError("session was not attached in time")

    def finish(self) -> None:
        with self._cv:
            self.lifecycle = Lifecycle.FINISHED
            self._cv.notify_all()

    def close(self, reason: str) -> None:
        audit("session_close", session=self.session_id, reason=reason)
        with self._cv:
            if self.lifecycle not in (Lifecycle.FINISHED,):
                self.failure = reason
                self.lifecycle = Lifecycle.FAILED
            self._cv.notify_all()

    @property
    def done(self) -> bool:
        return self.lifecycle in (Lifecycle.DRAINED, Lifecycle.FINISHED)

    def _check(self) -> None:
        if self.failure is not None:
            raise SessionError(f"session {self.session_id} failed: {self.failure}")


class SessionManager:
    """Owns sessions; a watchdog fails sessions not attached within the timeout."""

    def __init__(self, attach_timeout: float = 30.0, sweep_s: float = 0.5):
        self.attach_timeout = attach_timeout
        self._sessions: dict[str, Session] = {}
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._watch, args=(sweep_s,), daemon=True, name="kvbm-sessions")
        self._t.start()

    def open(self, initiator: int, holder: int) -> Session:
        s = Session(initiator=initiator, holder=holder)
        with self._lock:
            self._sessions[s.session_id] = s
        return s

    def get(self, sid: str) -> Session:
        with self._lock:
            return self._sessions[sid]

    def remove(self, sid: str) -> None:
        with self._lock:
            self._sessions.pop(sid, None)

    def _watch(self, sweep_s):
        while not self._stop.wait(sweep_s):
            now = time.monotonic()
            with self._lock:
                stale = [s for s in self._sessions.values()
                         if not s.attached and s.failure is None and now - s.created > self.attach_timeout]
                for s in stale:
                    del self._sessions[s.session_id]
            for s in stale:
                s.close("attach timeout")

    def __len__(self):
        with self._lock:
            return len(self._sessions)

    def close(self):
        self._stop.set()
        self._t.join(timeout=2)
