"""Branch-point tracking, registration handles with typed attachments, and
per-request block assignments (CPU)."""

import pytest

from kvbm_b200.logical.assignments import (DuplicateBlockId, ExternalBlockAssignments, LogicalBlockAssignments,
                                           OrderingViolation, PositionMismatch, SequenceHashMismatch, zip_assigned,
                                           zip_assigned_pending)
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.registry import (AttachmentError, BlockRegistry, BranchPointTracker, branch_points_on_prefix,
                                        hot_branch_points, is_branch_hash)
from kvbm_b200.logical.sequence import lineage, position, sequence_hashes


def chain(tokens, bs=1):
    return sequence_hashes(tokens, bs)


# ------------------------------------------------------------------ branch points
def test_linear_chain_has_no_branch_points():
    t = BranchPointTracker(1024)
    for h in chain(list(range(5))):
        t.on_block_registered(h)
    assert t.branch_point_count() == 0 and t.tracked_parent_count() == 4
    assert not any(is_branch_hash(t, h) for h in chain(list(range(5))))


def test_fork_is_detected_at_the_shared_parent():
    t = BranchPointTracker(1024)
    a, b = chain([0, 1, 2]), chain([0, 1, 99])
    for h in a + b:
        t.on_block_registered(h)
    assert a[:2] == b[:2] and a[2] != b[2]
    [(pos, frag, fan)] = t.current_branch_points()
    assert (pos, frag, fan) == (1, lineage(a[1]), 2)
    assert is_branch_hash(t, a[1]) and t.current_fanout(1, lineage(a[1])) == 2
    assert t.current_fanout(2, lineage(a[2])) is None  # leaves have no children
    # registering a duplicate child does not change the fanout
    t.on_block_registered(b[2])
    assert t.current_fanout(1, lineage(a[1])) == 2
    [rec] = hot_branch_points(t, 10)
    assert rec.position == 1 and rec.max_fanout == 2 and rec.observation_count == 1
    on = branch_points_on_prefix(t, a)
    assert [r.position for r in on] == [1]


def test_fanout_grows_and_history_is_bounded():
    t = BranchPointTracker(2)
    base = [5, 6, 7]
    for tail in range(4):
        for h in chain(base + [100 + tail]):
            t.on_block_registered(h)
    root = chain(base)[-1]
    assert t.current_fanout(position(root), lineage(root)) == 4
    [rec] = hot_branch_points(t, 5)
    assert rec.current_fanout == 4 and rec.max_fanout == 4 and rec.observation_count == 3
    # three more independent forks: history keeps at most two records, live state keeps all four
    for k in range(3):
        for tail in (1, 2):
            for h in chain([50 + k, 60 + k, tail]):
                t.on_block_registered(h)
    assert t.branch_point_count() == 4 and t.history_len() == 2


def test_registry_feeds_the_tracker_on_first_presence():
    reg = BlockRegistry(branch_history=64)
    g2 = BlockManager(16, 4, "lru", Tier.G2, registry=reg)
    g3 = BlockManager(16, 4, "lru", Tier.G3, registry=reg)
    a = sequence_hashes(list(range(12)), 4)
    b = sequence_hashes(list(range(8)) + [90, 91, 92, 93], 4)
    held = g2.register_mutable(g2.allocate_blocks(3), a) + g2.register_mutable(g2.allocate_blocks(1), b[2:])
    held += g3.register_mutable(g3.allocate_blocks(3), a)  # same hashes in another tier: no new children
    tr = reg.branch_tracker
    assert tr.branch_point_count() == 1 and tr.current_fanout(1, lineage(a[1])) == 2
    assert tr.tick == 3  # one per non-root registration
    del held


# -------------------------------------------------------------- registration handles
class OffloadMark:
    def __init__(self, n):
        self.n = n


def test_handles_are_shared_and_carry_typed_attachments():
    reg = BlockRegistry()
    g2 = BlockManager(8, 4, "lru", Tier.G2, registry=reg)
    g3 = BlockManager(8, 4, "lru", Tier.G3, registry=reg)
    hs = sequence_hashes(list(range(8)), 4)
    blocks = g2.register_mutable(g2.allocate_blocks(2), hs)
    h = blocks[0].registration_handle()
    assert h is g2.registration_handle(hs[0]) and h.is_from_registry(reg)
    assert h.has_block(Tier.G2) and not h.has_block(Tier.G3) and h.tiers() == [Tier.G2]
    copy = g3.register_mutable(g3.allocate_blocks(1), hs[:1])
    assert h.has_any_block([Tier.G3]) and h.tiers() == [Tier.G2, Tier.G3]
    h.attach_unique(OffloadMark(1))
    h.attach_unique(OffloadMark(2))  # unique replaces
    assert h.get(OffloadMark).unique().n == 2
    h.attach("router-a", key=str)
    h.attach("router-b", key=str)
    assert h.get(str).multiple() == ["router-a", "router-b"]
    with pytest.raises(AttachmentError):
        h.attach(OffloadMark(3))
    with pytest.raises(AttachmentError):
        h.attach_unique("x", key=str)
    assert h.get(OffloadMark).with_all(lambda u, m: (u.n, m)) == (2, [])
    assert h.get(OffloadMark).replace_unique(lambda v: OffloadMark(v.n + 1)) and h.get(OffloadMark).unique().n == 3
    seen = []
    h.on_touch(seen.append)
    h.touch()
    assert seen == [hs[0]]
    assert g3.registration_handle(hs[0]) is h  # one handle per hash across tiers
    assert reg.handle(12345) is None


def test_handles_drop_once_no_tier_holds_the_hash():
    reg = BlockRegistry()
    g2 = BlockManager(4, 4, "lru", Tier.G2, registry=reg)
    hs = sequence_hashes(list(range(4)), 4)
    [b] = g2.register_mutable(g2.allocate_blocks(1), hs)
    reg.handle(hs[0]).attach_unique(OffloadMark(7))
    b.release()
    assert reg.handle(hs[0]).get(OffloadMark).unique().n == 7  # inactive but still registered
    g2.reset_inactive_pool()
    assert reg.handle(hs[0]) is None and len(reg) == 0
    [b2] = g2.register_mutable(g2.allocate_blocks(1), hs)
    assert reg.handle(hs[0]).get(OffloadMark).unique() is None  # a new registration starts empty
    assert reg.prune() == 0
    b2.release()


# ------------------------------------------------------------------ assignments
def test_external_assignments_lifecycle_and_zips():
    hs = sequence_hashes(list(range(40)), 4)  # 10 blocks
    g2 = ExternalBlockAssignments(offset=0)
    g2.extend_block_ids([100, 101, 102, 103])
    assert g2.pending_positions() == range(0, 4)
    assert g2.assign_pending(hs) == range(0, 4)
    assert [h for _, h in g2.assigned_iter()] == hs[:4]
    g1 = ExternalBlockAssignments(offset=0)
    g1.extend_assigned([(7, hs[0])])
    g1.extend_block_ids([7, 8, 9, 10, 11, 12])  # known prefix skipped, the rest pending
    assert g1.pending_positions() == range(1, 6)
    assert zip_assigned_pending(g2, g1) == [(1, 101, 8), (2, 102, 9), (3, 103, 10)]
    assert g1.stage_pending(hs) == range(0, 5) and g1.staged_positions() == range(1, 6)
    assert g1.commit_staged() == range(1, 6)
    assert zip_assigned(g2, g1) == [(0, 100, 7), (1, 101, 8), (2, 102, 9), (3, 103, 10)]
    with pytest.raises(OrderingViolation):
        g1.extend_block_ids([200, 7])
    with pytest.raises(DuplicateBlockId):
        g1.extend_block_ids([300, 300])
    assert g1.unassigned_count() == 0  # failed calls changed nothing


def test_external_assignments_with_offset_and_position_check():
    hs = sequence_hashes(list(range(40)), 4)
    g3 = ExternalBlockAssignments(offset=6)
    g3.extend_block_ids([1, 2, 3, 4, 5])
    assert g3.assign_pending(hs) == range(0, 4)  # positions 6..9 (only ten blocks exist)
    assert g3.get_at_position(6) == (1, hs[6]) and g3.get_pending_at_position(10) == 5
    bad = ExternalBlockAssignments(offset=2)
    bad.extend_block_ids([9])
    with pytest.raises(PositionMismatch):
        bad.stage_pending([0, 0, hs[5]])  # position 5 hash offered for position 2
    assert bad.unassigned_count() == 1


def test_logical_assignments_stage_register_and_release():
    mgr = BlockManager(8, 4, "lru", Tier.G1)
    hs = sequence_hashes(list(range(12)), 4)
    la = LogicalBlockAssignments()
    blocks = mgr.allocate_blocks(3)
    assert la.extend_blocks(blocks) == 3
    with pytest.raises(DuplicateBlockId) as e:
        la.extend_blocks([blocks[0]])
    assert e.value.blocks == [blocks[0]]
    assert la.stage(hs[:2]) == 2 and la.staged_count() == 2 and la.unassigned_count() == 1
    assert la.register(mgr) == 2 and la.sequence_hashes() == hs[:2]
    assert mgr.active_len() == 2
    matched = mgr.match_blocks(hs)
    other = LogicalBlockAssignments()
    with pytest.raises(SequenceHashMismatch):
        other.extend_assigned(matched, expected_hashes=[hs[1], hs[0]])
    other.extend_assigned(matched, expected_hashes=hs)
    assert other.assigned_count() == 2
    other.clear()
    bid, last = la.pop_last_unassigned()
    assert bid == blocks[2].block_id
    last.release()
    la.clear()
    assert la.is_empty() and mgr.active_len() == 0 and mgr.inactive_len() == 2


def test_token_sequence_incremental_hashes_match_one_shot():
    """Appending one token at a time, in chunks, or after a truncation gives the same block hashes
    as hashing the whole token list at once (the buffer grows by doubling)."""
    import numpy as np

    from kvbm_b200.logical.sequence import TokenBlockSequence, sequence_hashes

    rng = np.random.default_rng(3)
    toks = rng.integers(0, 50000, 700).tolist()
    for salt in (None, "lora-a"):
        want = sequence_hashes(toks, 16, salt)
        s = TokenBlockSequence(toks[:5], 16, salt)
        i = 5
        while i < len(toks):
            k = int(rng.integers(1, 40))
            if k == 1:
                new = s.append(np.int64(toks[i]))
            else:
                new = s.append(toks[i: i + k])
            i += k
            assert all(h in want for h in new)
        assert s.sequence_hashes == want and len(s) == len(toks) and list(s.tokens) == toks
        assert list(s.partial_tokens) == toks[len(want) * 16:]
        s.truncate(333)
        assert s.sequence_hashes == want[: 333 // 16] and len(s) == 333
        s.append(toks[333:])
        assert s.sequence_hashes == want
