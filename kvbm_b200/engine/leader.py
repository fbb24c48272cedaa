"""InstanceLeader: the logical owner of an instance's G2/G3 (and G4) tiers.

The leader answers "how much of this sequence is cached below G1?" and
decides onboards and offloads; its workers move the bytes.

* ``find_matches`` walks the G2 pool (prefix match, references taken), then
  continues in G3 from where G2 stopped, then in the object store (G4, an
  ``engine.object_tier.ObjectTier``). G3 and G4 hits are staged into G2
  unless the staging mode says to only hold or prepare them.
* ``onboard`` copies matched G2 blocks into framework-owned G1 block ids on
  every worker (whole blocks, or layer by layer).
* ``offload`` queues G1 blocks for the G1 -> G2 pipeline (and, by chaining,
  G2 -> G3 / G4).

Parity: crates/kvbm-engine/src/leader/{instance.rs:72-1592 (InstanceLeader,
scan_blocks, find/stage/pull), types.rs (StagingMode{Hold,Prepare,Full},
FindMatchesOptions, FindMatchesResult), onboarding.rs (OnboardingStatus)};
docs/leader.md:58-76.
"""

from __future__ import annotations

import enum
import threading
import uuid
from dataclasses import dataclass, field

from ..logical.manager import BlockManager, ImmutableBlock, Tier
from ..physical.transfer import TransferCompleteNotification
from .offload import OffloadEngine, OffloadHandle, OffloadItem


class StagingMode(str, enum.Enum):
    HOLD = "hold"        # report G3 hits, keep them in G3
    PREPARE = "prepare"  # take references on G3 hits, stage later
    FULL = "full"        # stage G3 hits into G2 now


class OnboardingStatus(str, enum.Enum):
    SEARCHING = "searching"
    STAGING = "staging"
    READY = "ready"
    ONBOARDING = "onboarding"
    COMPLETE = "complete"
    FAILED = "failed"


@dataclass
class FindMatchesOptions:
    staging: StagingMode = StagingMode.FULL
    search_remote: bool = False


@dataclass
class FindMatchesResult:
    g2_blocks: list[ImmutableBlock] = field(default_factory=list)
    g3_held: list[ImmutableBlock] = field(default_factory=list)
    staged_from_g3: int = 0
    status: OnboardingStatus = OnboardingStatus.READY

    @property
    def num_blocks(self) -> int:
        return len(self.g2_blocks) + len(self.g3_held)

    def release(self) -> None:
        for b in self.g2_blocks + self.g3_held:
            b.release()
        self.g2_blocks, self.g3_held = [], []


class ParallelWorkers:
    """Fan a transfer out to every worker (TP ranks each hold their head shard)."""

    def __init__(self, workers: list):
        self.workers = list(workers)

    def execute_local_transfer(self, src_tier, src_ids, dst_tier, dst_ids, layer_range=None):
        notes = [w.execute_local_transfer(src_tier, src_ids, dst_tier, dst_ids, layer_range=layer_range)
                 for w in self.workers]
        return TransferCompleteNotification.aggregate(notes)

    def start_layerwise_onboard(self, g2_ids, g1_ids) -> None:
        for w in self.workers:
            w.start_layerwise_onboard(g2_ids, g1_ids)

    def __len__(self):
        return len(self.workers)


class InstanceLeader:
    def __init__(self, g2: BlockManager, workers: ParallelWorkers, g3: BlockManager | None = None,
                 offload: OffloadEngine | None = None, object_store=None, instance_id: int | None = None):
        self.g2, self.g3, self.workers = g2, g3, workers
        self.offload_engine = offload
        self.object_store = object_store
        self.instance_id = instance_id if instance_id is not None else uuid.uuid4().int
        self._lock = threading.Lock()
        self.stats = {"find_calls": 0, "g2_hits": 0, "g3_hits": 0, "onboarded_blocks": 0, "offloaded_blocks": 0}

    @classmethod
    def scheduler_side(cls, g2: BlockManager, g3: BlockManager | None = None, **kw) -> "InstanceLeader":
        """The leader a connector's scheduler process holds: it owns the G2/G3 pools'
        logical state (matching, registration, eviction) while the bytes are moved by
        the connector's workers in the model-runner processes, which receive their
        onboard / offload / stage / spill ops in the per-step connector metadata. It
        has no in-process workers, so a direct ``onboard`` or ``stage_g3_to_g2``
        raises instead of silently moving nothing."""
        return cls(g2, ParallelWorkers([]), g3=g3, **kw)

    # --------------------------------------------------------------- find
    def find_matches(self, seq_hashes: list[int], options: FindMatchesOptions | None = None) -> FindMatchesResult:
        opts = options or FindMatchesOptions()
        self.stats["find_calls"] += 1
        res = FindMatchesResult(g2_blocks=self.g2.match_blocks(seq_hashes))
        self.stats["g2_hits"] += len(res.g2_blocks)
        rest = seq_hashes[len(res.g2_blocks):]
        if self.g3 is None or not rest:
            return self._find_g4(res, rest, opts)
        if opts.staging == StagingMode.HOLD:
            n = self.g3.count_prefix(rest)
            self.stats["g3_hits"] += n
            res.status = OnboardingStatus.READY if n == 0 else OnboardingStatus.STAGING
            res.g3_held = []
            res.staged_from_g3 = 0
            res._g3_count = n  # type: ignore[attr-defined]
            return res
        g3_hits = self.g3.match_blocks(rest)
        self.stats["g3_hits"] += len(g3_hits)
        if not g3_hits:
            return self._find_g4(res, rest, opts)
        if opts.staging == StagingMode.PREPARE:
            res.g3_held = g3_hits
            res.status = OnboardingStatus.STAGING
            return res
        staged = self.stage_g3_to_g2(g3_hits)
        res.g2_blocks += staged
        res.staged_from_g3 = len(g3_hits)
        if len(staged) == len(g3_hits):
            return self._find_g4(res, rest[len(g3_hits):], opts)
        return res

    def _find_g4(self, res: FindMatchesResult, rest: list[int], opts: FindMatchesOptions) -> FindMatchesResult:
        """Continue a find in the object store (G4 -> G2) when one is attached and staging is FULL."""
        if self.object_store is None or not rest or opts.staging != StagingMode.FULL:
            return res
        staged = self.object_store.stage(rest, self.g2)
        self.stats["g4_hits"] = self.stats.get("g4_hits", 0) + len(staged)
        res.g2_blocks += staged
        res.staged_from_g4 = len(staged)  # type: ignore[attr-defined]
        return res

    def stage_g3_to_g2(self, g3_blocks: list[ImmutableBlock]) -> list[ImmutableBlock]:
        """Disk -> pinned for the given G3 blocks; returns the registered G2 blocks.

        The copy runs on this leader's workers; a leader without workers (the
        scheduler side of a connector, whose workers live in other processes)
        cannot stage and raises: it finds with ``StagingMode.PREPARE`` and has
        the connector's workers stage the held blocks with the onboard."""
        if not len(self.workers):
            for b in g3_blocks:
                b.release()
            raise RuntimeError("no workers to stage G3 -> G2 here; find with StagingMode.PREPARE and let the "
                               "connector's workers stage the held G3 blocks")
        got = self.g2.allocate_blocks_with_evictions(len(g3_blocks))
        if got is None:
            for b in g3_blocks:
                b.release()
            return []
        dst, _ = got
        note = self.workers.execute_local_transfer(Tier.G3, [b.block_id for b in g3_blocks], Tier.G2,
                                                   [d.block_id for d in dst])
        note.wait()
        staged = self.g2.register_mutable(dst, [b.sequence_hash for b in g3_blocks])
        for b in g3_blocks:
            b.release()
        return staged

    def scan_blocks(self, seq_hashes: list[int], tier: Tier = Tier.G2, touch: bool = False) -> dict[int, ImmutableBlock]:
        mgr = {Tier.G2: self.g2, Tier.G3: self.g3}[Tier(tier)]
        return {} if mgr is None else mgr.scan_matches(seq_hashes, touch)

    # ------------------------------------------------------------ onboard
    def onboard(self, g2_blocks: list[ImmutableBlock], g1_block_ids: list[int],
                layerwise: bool = False) -> TransferCompleteNotification | None:
        if len(g2_blocks) != len(g1_block_ids):
            raise ValueError("one G1 destination per G2 block")
        if not g2_blocks:
            return TransferCompleteNotification.ready()
        if not len(self.workers):
            raise RuntimeError("this leader has no in-process workers; onboards travel to the connector's "
                               "workers in the step's connector metadata")
        ids = [b.block_id for b in g2_blocks]
        self.stats["onboarded_blocks"] += len(ids)
        if layerwise:
            self.workers.start_layerwise_onboard(ids, list(g1_block_ids))
            return None
        return self.workers.execute_local_transfer(Tier.G2, ids, Tier.G1, list(g1_block_ids))

    # ------------------------------------------------------------ offload
    def offload_g1(self, seq_hashes: list[int], g1_block_ids: list[int], precondition=None) -> OffloadHandle:
        if self.offload_engine is None:
            raise RuntimeError("no offload engine configured")
        items = [OffloadItem(h, b) for h, b in zip(seq_hashes, g1_block_ids)]
        self.stats["offloaded_blocks"] += len(items)
        return self.offload_engine.enqueue_g1_to_g2_with_precondition(items, precondition)
