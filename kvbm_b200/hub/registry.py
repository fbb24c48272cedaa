"""Hub instance registry with heartbeat TTL.

Connector leaders register (instance id, control address, worker peers,
feature set, layout facts); each registration must be refreshed by a
heartbeat within ``ttl`` seconds or it is evicted, and eviction removes the
instance from the indexer and the prefill router too.

Parity: crates/kvbm-hub/src/registry.rs (TTL 30 s default :199-206,
100 ms in tests :421-440), handlers.rs (heartbeat, probe),
protocol.rs:30-81 (paths).
"""

from __future__ import annotations

import threading
import time
from dataclasses import asdict, dataclass, field
from typing import Callable


@dataclass
class InstanceRecord:
    instance_id: int
    address: str = ""
    role: str = "both"                      # prefill | decode | both
    features: list[str] = field(default_factory=list)
    workers: dict[str, str] = field(default_factory=dict)  # worker id -> messenger address
    block_size: int = 16
    max_seq_len: int | None = None
    layout: dict = field(default_factory=dict)
    last_seen: float = field(default_factory=time.monotonic)
    registered_at: float = field(default_factory=time.time)

    def public(self) -> dict:
        d = asdict(self)
        d["instance_id"] = str(self.instance_id)
        d.pop("last_seen")
        return d


class InstanceRegistry:
    def __init__(self, ttl: float = 30.0, on_evict: Callable[[int], None] | None = None):
        self.ttl = ttl
        self.on_evict = on_evict
        self._items: dict[int, InstanceRecord] = {}
        self._lock = threading.Lock()

    def register(self, rec: InstanceRecord) -> InstanceRecord:
        rec.last_seen = time.monotonic()
        with self._lock:
            self._items[rec.instance_id] = rec
        return rec

    def heartbeat(self, instance_id: int) -> bool:
        with self._lock:
            rec = self._items.get(instance_id)
            if rec is None:
                return False
            rec.last_seen = time.monotonic()
            return True

    def unregister(self, instance_id: int) -> bool:
        with self._lock:
            gone = self._items.pop(instance_id, None)
        if gone is not None and self.on_evict:
            self.on_evict(instance_id)
        return gone is not None

    def sweep(self) -> list[int]:
        now = time.monotonic()
        with self._lock:
            dead = [i for i, r in self._items.items() if now - r.last_seen > self.ttl]
            for i in dead:
                del self._items[i]
        for i in dead:
            if self.on_evict:
                self.on_evict(i)
        return dead

    def get(self, instance_id: int) -> InstanceRecord | None:
        with self._lock:
            return self._items.get(instance_id)

    def list(self, role: str | None = None, feature: str | None = None) -> list[InstanceRecord]:
        with self._lock:
            recs = list(self._items.values())
        if role:
            recs = [r for r in recs if r.role in (role, "both")]
        if feature:
            recs = [r for r in recs if feature in r.features]
        return recs

    def peer_by_worker(self, worker_id: str) -> tuple[int, str] | None:
        with self._lock:
            for r in self._items.values():
                if worker_id in r.workers:
                    return r.instance_id, r.workers[worker_id]
        return None
