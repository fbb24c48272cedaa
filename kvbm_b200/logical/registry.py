"""Registration handles, typed attachments and branch-point tracking.

``BlockRegistry`` is the Python face of the native cross-tier registry
(per-hash presence counts per tier, KV events, TinyLFU frequencies, branch
points). It hands out one :class:`RegistrationHandle` per sequence hash:
callers ask for the handle of a registered block and hang their own data on
it (``attach_unique`` / ``attach``, keyed by the value's type), register
touch callbacks, or ask which tiers hold the block (``has_block``). Every
caller that asks for the same hash while it is registered gets the same
handle object, so attachments made by one component (an offload policy, a
remote-search index, a router) are visible to the others. The registry keeps
a handle while its hash is present in some tier; ``prune`` (also run
automatically as the table grows) drops the handles of hashes that left every
tier, with their attachments - the lifetime the reference gives the handle by
tying it to the registered blocks that hold it.

``BranchPointTracker`` is the native tracker: every hash that becomes
present in a registry with a tracker updates the parent node's set of
distinct children; a node with more than one child is a branch point.

Parity: crates/kvbm-logical/src/registry/handle.rs:27-258
(BlockRegistrationHandle: seq_hash, is_from_registry, has_block,
has_any_block, on_touch, touch, get, attach_unique, attach),
registry/attachments.rs:14-170 (AttachmentError, TypedAttachments
with_unique / with_multiple / with_all and their _mut forms),
branch_tracker.rs:189-345 (BranchPointTracker).
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Any, Callable, Iterable, Sequence

from .. import _core_native as core
from .manager import Tier
from .sequence import lineage, position

BranchPointTracker = core.BranchTracker


@dataclass(frozen=True)
class BranchPointRecord:
    """A branch point: the node at ``position`` whose lineage is ``fragment``."""

    position: int
    fragment: int
    current_fanout: int
    max_fanout: int
    observation_count: int
    last_updated_tick: int

    @classmethod
    def from_native(cls, d: dict) -> "BranchPointRecord":
        return cls(**d)


def hot_branch_points(tracker, limit: int) -> list[BranchPointRecord]:
    return [BranchPointRecord.from_native(d) for d in tracker.hot_branch_points(limit)]


def branch_points_on_prefix(tracker, prefix: Sequence[int]) -> list[BranchPointRecord]:
    """Branch points along a prefix of sequence hashes (hash i at block position i)."""
    return [BranchPointRecord.from_native(d) for d in tracker.branch_points_on_prefix(list(prefix))]


def is_branch_hash(tracker, seq_hash: int) -> bool:
    """True when the block named by ``seq_hash`` has more than one distinct registered child."""
    return tracker.is_branch_point(position(seq_hash), lineage(seq_hash))


class AttachmentError(TypeError):
    """A type was attached as unique and then as multiple, or the other way round."""


class TypedAttachments:
    """The attachments of one type on one handle."""

    def __init__(self, handle: "RegistrationHandle", key: type):
        self._h, self._key = handle, key

    def unique(self) -> Any | None:
        with self._h._lock:
            return self._h._unique.get(self._key)

    def multiple(self) -> list:
        with self._h._lock:
            return list(self._h._multiple.get(self._key, ()))

    def with_unique(self, fn: Callable[[Any], Any]):
        """``fn(value)`` under the handle's lock when a unique value is attached, else None."""
        with self._h._lock:
            if self._key not in self._h._unique:
                return None
            return fn(self._h._unique[self._key])

    def with_multiple(self, fn: Callable[[list], Any]):
        with self._h._lock:
            return fn(self._h._multiple.get(self._key, []))

    def with_all(self, fn: Callable[[Any | None, list], Any]):
        with self._h._lock:
            return fn(self._h._unique.get(self._key), self._h._multiple.get(self._key, []))

    def replace_unique(self, fn: Callable[[Any], Any]) -> bool:
        """Swap the unique value for ``fn(value)``; False when none is attached."""
        with self._h._lock:
            if self._key not in self._h._unique:
                return False
            self._h._unique[self._key] = fn(self._h._unique[self._key])
            return True


class RegistrationHandle:
    """The identity of one registered sequence hash, shared by every holder of the block."""

    __slots__ = ("seq_hash", "_registry", "_lock", "_unique", "_multiple", "_mode", "_touch", "__weakref__")

    def __init__(self, seq_hash: int, registry: "BlockRegistry"):
        self.seq_hash = int(seq_hash)
        self._registry = registry
        self._lock = threading.Lock()
        self._unique: dict[type, Any] = {}
        self._multiple: dict[type, list] = {}
        self._mode: dict[type, str] = {}
        self._touch: list[Callable[[int], None]] = []

    @property
    def position(self) -> int:
        return position(self.seq_hash)

    def is_from_registry(self, registry: "BlockRegistry") -> bool:
        return self._registry is registry

    # ---------------------------------------------------------- presence
    def has_block(self, tier: Tier | int) -> bool:
        """True while a block of ``tier`` holds this hash (primary or duplicate)."""
        return bool(self._registry.native.is_present(self.seq_hash, int(tier)))

    def has_any_block(self, tiers: Iterable[Tier | int]) -> bool:
        mask = self._registry.native.presence_mask(self.seq_hash)
        return any(mask >> int(t) & 1 for t in tiers)

    def tiers(self) -> list[Tier]:
        mask = self._registry.native.presence_mask(self.seq_hash)
        return [t for t in Tier if mask >> int(t) & 1]

    # ------------------------------------------------------------- touch
    def on_touch(self, callback: Callable[[int], None]) -> None:
        with self._lock:
            self._touch.append(callback)

    def touch(self) -> None:
        """Count one access in the registry's frequency sketch and run the touch callbacks
        (outside the handle's lock, so a callback may use the handle)."""
        self._registry.native.touch(self.seq_hash)
        with self._lock:
            cbs = list(self._touch)
        for cb in cbs:
            cb(self.seq_hash)

    # ------------------------------------------------------- attachments
    def get(self, key: type) -> TypedAttachments:
        return TypedAttachments(self, key)

    def attach_unique(self, value: Any, key: type | None = None) -> None:
        """Attach ``value`` as the one value of its type (replacing an earlier one)."""
        key = type(value) if key is None else key
        with self._lock:
            if self._mode.get(key) == "multiple":
                raise AttachmentError(f"{key.__name__} is already attached as multiple")
            self._unique[key] = value
            self._mode[key] = "unique"

    def attach(self, value: Any, key: type | None = None) -> None:
        """Add ``value`` to the list of values of its type."""
        key = type(value) if key is None else key
        with self._lock:
            if self._mode.get(key) == "unique":
                raise AttachmentError(f"{key.__name__} is already attached as unique")
            self._multiple.setdefault(key, []).append(value)
            self._mode[key] = "multiple"

    def detach(self, key: type) -> None:
        with self._lock:
            self._unique.pop(key, None)
            self._multiple.pop(key, None)
            self._mode.pop(key, None)

    def __repr__(self):
        return f"RegistrationHandle(pos={self.position}, {self.seq_hash & 0xFFFFFFFFFFFFFFFF:#x})"


class BlockRegistry:
    """The registry shared by the block managers of every tier of one instance.

    ``BlockRegistry(branch_history=1024)`` also tracks branch points; pass ``native`` to wrap a
    registry that already exists (its events, frequency sketch and tracker stay as they are)."""

    def __init__(self, native=None, events=None, frequency=None, branch_history: int | None = None):
        if native is None:
            tracker = core.BranchTracker(branch_history) if branch_history is not None else None
            native = core.Registry(events=events, frequency=frequency, branch_tracker=tracker)
        self.native = native
        self._handles: dict[int, RegistrationHandle] = {}
        self._lock = threading.Lock()
        self._prune_at = 1024

    @property
    def branch_tracker(self):
        return self.native.branch_tracker

    def is_registered(self, seq_hash: int, tier: Tier | int = -1) -> bool:
        return bool(self.native.is_present(int(seq_hash), int(tier)))

    def handle(self, seq_hash: int) -> RegistrationHandle | None:
        """The handle of a hash present in some tier (created on first request), else None."""
        seq_hash = int(seq_hash)
        if not self.native.is_present(seq_hash, -1):
            with self._lock:
                self._handles.pop(seq_hash, None)
            return None
        with self._lock:
            h = self._handles.get(seq_hash)
            if h is None:
                h = self._handles[seq_hash] = RegistrationHandle(seq_hash, self)
                if len(self._handles) >= self._prune_at:
                    self._prune_locked()
            return h

    def prune(self) -> int:
        """Drop the handles (and attachments) of hashes no tier holds any more; returns how many."""
        with self._lock:
            return self._prune_locked()

    def _prune_locked(self) -> int:
        gone = [k for k in self._handles if not self.native.is_present(k, -1)]
        for k in gone:
            del self._handles[k]
        self._prune_at = max(1024, 2 * len(self._handles))
        return len(gone)

    def __len__(self) -> int:
        with self._lock:
            return len(self._handles)
