"""Typed block lifecycle over the C++ BlockPool.

Python objects give the reference's type-state guarantees at run time:
``MutableBlock`` (allocated, writable) -> ``CompleteBlock`` (full, staged
under a sequence hash) -> ``ImmutableBlock`` (registered, shareable,
reference counted). Dropping the last handle of a block returns it to the
pool: a mutable or staged block goes back to the reset pool, a registered
primary moves to the inactive (evictable, still matchable) pool.

Parity: crates/kvbm-logical/src/manager/mod.rs:31-230 (BlockManager:
allocate_blocks, allocate_blocks_with_evictions, reset_inactive_pool,
register_blocks, match_blocks, scan_matches, total/available_blocks),
blocks/{mutable,complete,immutable}.rs (type states), manager/builder.rs
(block_size default 16, default inactive backend lineage/tick).
"""

from __future__ import annotations

import enum
import threading
from typing import Iterable, Sequence

from .. import _core_native as core


class Tier(enum.IntEnum):
    """Storage tiers (the reference's zero-sized G1..G4 markers)."""

    G1 = 0  # device HBM
    G2 = 1  # pinned host
    G3 = 2  # local disk
    G4 = 3  # object store


class BlockManagerResetError(RuntimeError):
    pass


class _Handle:
    __slots__ = ("_mgr", "block_id", "_live")

    def __init__(self, mgr: "BlockManager", block_id: int):
        self._mgr = mgr
        self.block_id = block_id
        self._live = True

    def _take(self) -> None:
        if not self._live:
            raise RuntimeError(f"{type(self).__name__} {self.block_id} already consumed")
        self._live = False

    @property
    def tier(self) -> Tier:
        return self._mgr.tier


class MutableBlock(_Handle):
    """An allocated block that can be filled. Dropping it resets the slot."""

    __slots__ = ()

    def complete(self, sequence_hash: int) -> "CompleteBlock":
        self._take()
        self._mgr._pool.stage(self.block_id, sequence_hash)
        return CompleteBlock(self._mgr, self.block_id, sequence_hash)

    stage = complete

    def release(self) -> None:
        if self._live:
            self._live = False
            self._mgr._pool.release_mutable(self.block_id)

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def __repr__(self):
        return f"MutableBlock({self.block_id})"


class CompleteBlock(_Handle):
    """A full block staged under its sequence hash, ready to register."""

    __slots__ = ("sequence_hash",)

    def __init__(self, mgr, block_id, sequence_hash):
        super().__init__(mgr, block_id)
        self.sequence_hash = sequence_hash

    def reset(self) -> MutableBlock:
        self._take()
        self._mgr._pool.unstage(self.block_id)
        return MutableBlock(self._mgr, self.block_id)

    def release(self) -> None:
        if self._live:
            self._live = False
            self._mgr._pool.release_staged(self.block_id)

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def __repr__(self):
        return f"CompleteBlock({self.block_id}, {self.sequence_hash:#x})"


class ImmutableBlock(_Handle):
    """A registered block; each handle holds one reference."""

    __slots__ = ("sequence_hash", "kind")

    def __init__(self, mgr, block_id, sequence_hash, kind: str = "primary"):
        # the base initialiser inlined: a prefix match builds one handle per hit
        self._mgr = mgr
        self.block_id = block_id
        self._live = True
        self.sequence_hash = sequence_hash
        self.kind = kind

    def clone(self) -> "ImmutableBlock":
        if not self._live:
            raise RuntimeError("released block")
        self._mgr._pool.add_ref(self.block_id)
        return ImmutableBlock(self._mgr, self.block_id, self.sequence_hash, self.kind)

    def registration_handle(self):
        return self._mgr.registration_handle(self.sequence_hash)

    def downgrade(self) -> "WeakBlock":
        return WeakBlock(self._mgr, self.sequence_hash)

    def release(self) -> None:
        if self._live:
            self._live = False
            self._mgr._pool.release(self.block_id)

    def set_reset_on_release(self, value: bool = True) -> None:
        self._mgr._pool.set_reset_on_release(self.block_id, value)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def __repr__(self):
        return f"ImmutableBlock({self.block_id}, {self.sequence_hash:#x}, {self.kind})"


class WeakBlock:
    """A non-owning reference: upgrade() re-acquires the block if it is still cached."""

    __slots__ = ("_mgr", "sequence_hash")

    def __init__(self, mgr, sequence_hash):
        self._mgr, self.sequence_hash = mgr, sequence_hash

    def upgrade(self) -> ImmutableBlock | None:
        got = self._mgr.match_blocks([self.sequence_hash])
        return got[0] if got else None


class BlockManager:
    """Block pool of one tier with sequence-hash prefix reuse."""

    def __init__(self, num_blocks: int, block_size: int = 16, inactive: str = "lineage", tier: Tier = Tier.G2,
                 registry: "core.Registry | None" = None, duplicate_policy: str = "allow", events=None,
                 frequency: "core.TinyLfu | None" = None):
        if registry is None:
            if frequency is None and inactive == "multi_lru":
                frequency = core.TinyLfu()
            registry = core.Registry(events=events, frequency=frequency)
        # a logical.registry.BlockRegistry (handles, attachments) or a bare native registry
        self.handles = registry if hasattr(registry, "native") else None
        registry = getattr(registry, "native", registry)
        self.tier = Tier(tier)
        self.registry = registry
        self._pool = core.BlockPool(num_blocks, block_size, inactive, int(self.tier), registry, duplicate_policy)
        self.duplicate_policy = duplicate_policy
        self._lock = threading.Lock()

    # ------------------------------------------------------------ allocate
    def allocate_blocks(self, count: int) -> list[MutableBlock] | None:
        got = self.allocate_blocks_with_evictions(count)
        return None if got is None else got[0]

    def allocate_blocks_with_evictions(self, count: int) -> tuple[list[MutableBlock], list[int]] | None:
        got = self._pool.allocate(count)
        if got is None:
            return None
        ids, evicted = got
        return [MutableBlock(self, i) for i in ids], evicted

    # ------------------------------------------------------------ register
    def register_block(self, block: CompleteBlock) -> ImmutableBlock:
        block._take()
        bid, kind = self._pool.register(block.block_id)
        k = {0: "primary", 1: "duplicate", 2: "primary"}[kind]
        return ImmutableBlock(self, bid, block.sequence_hash, k)

    def register_blocks(self, blocks: Iterable[CompleteBlock]) -> list[ImmutableBlock]:
        return [self.register_block(b) for b in blocks]

    def register_mutable(self, blocks: Sequence[MutableBlock], hashes: Sequence[int]) -> list[ImmutableBlock]:
        """complete() + register() for many blocks in one native call."""
        for b in blocks:
            b._take()
        res = self._pool.stage_and_register([b.block_id for b in blocks], list(hashes))
        return [ImmutableBlock(self, bid, h, "duplicate" if kind == 1 else "primary")
                for (bid, kind), h in zip(res, hashes)]

    def allocate_ids_with_evictions(self, count: int) -> list[int] | None:
        """Like ``allocate_blocks_with_evictions`` but returns bare ids, without a handle per block:
        the caller owns them and must hand every id back through ``register_ids`` /
        ``register_ids_released`` or ``release_ids`` (bulk paths of a scheduler)."""
        got = self._pool.allocate(count)
        return None if got is None else list(got[0])

    def release_ids(self, ids: Sequence[int]) -> None:
        """Return allocated, never-registered ids to the reset pool."""
        self._pool.release_mutable_many([int(i) for i in ids])

    def register_ids(self, ids: Sequence[int], hashes: Sequence[int]) -> list[ImmutableBlock]:
        """Register bare allocated ids under ``hashes``; one handle per registered block."""
        res = self._pool.stage_and_register([int(i) for i in ids], list(hashes))
        return [ImmutableBlock(self, bid, h, "duplicate" if kind == 1 else "primary")
                for (bid, kind), h in zip(res, hashes)]

    def register_ids_released(self, ids: Sequence[int], hashes: Sequence[int]) -> int:
        """Register bare allocated ids and release them at once: cached (inactive, matchable)."""
        res = self._pool.stage_and_register([int(i) for i in ids], list(hashes))
        self._pool.release_many([bid for bid, _ in res])
        return len(res)

    def register_mutable_released(self, blocks: Sequence[MutableBlock], hashes: Sequence[int]) -> int:
        """``register_mutable`` followed by releasing every handle, in two native calls: the
        blocks become cached (inactive, matchable) without a Python handle per block."""
        for b in blocks:
            b._take()
        res = self._pool.stage_and_register([b.block_id for b in blocks], list(hashes))
        self._pool.release_many([bid for bid, _ in res])
        return len(res)

    # --------------------------------------------------------------- match
    def match_blocks(self, seq_hashes: Sequence[int]) -> list[ImmutableBlock]:
        """Longest cached prefix of ``seq_hashes`` (stops at the first miss)."""
        ids = self._pool.match_prefix(list(seq_hashes))
        return [ImmutableBlock(self, i, h) for i, h in zip(ids, seq_hashes)]

    def scan_matches(self, seq_hashes: Sequence[int], touch: bool = False) -> dict[int, ImmutableBlock]:
        """Every cached block among ``seq_hashes`` (does not stop at a miss)."""
        found = self._pool.scan(list(seq_hashes), touch)
        return {h: ImmutableBlock(self, i, h) for h, i in found.items()}

    def count_prefix(self, seq_hashes: Sequence[int]) -> int:
        """Length of the cached prefix without taking references."""
        return self._pool.count_prefix(list(seq_hashes))

    def contains(self, seq_hash: int) -> bool:
        return self._pool.contains(seq_hash)

    def registration_handle(self, seq_hash: int):
        """The shared registration handle of a registered hash (managers built over a
        ``BlockRegistry``); None when the hash is not registered in any tier."""
        if self.handles is None:
            raise RuntimeError("this manager was built without a BlockRegistry")
        return self.handles.handle(seq_hash)

    # ---------------------------------------------------------------- admin
    def reset_inactive_pool(self) -> None:
        self._pool.reset_inactive()
        if self._pool.reset_len() != self.total_blocks():
            raise BlockManagerResetError(
                f"expected {self.total_blocks()} reset blocks, found {self._pool.reset_len()}")

    def total_blocks(self) -> int:
        return self._pool.total_blocks

    def available_blocks(self) -> int:
        return self._pool.available()

    def block_size(self) -> int:
        return self._pool.block_size

    def inactive_len(self) -> int:
        return self._pool.inactive_len()

    def reset_len(self) -> int:
        return self._pool.reset_len()

    def active_len(self) -> int:
        return self._pool.active_len()

    def metrics(self) -> dict:
        return self._pool.metrics()

    @property
    def native(self):
        return self._pool
