"""CPU tests of the C++ block pool: lifecycle, prefix match, eviction
policies, duplicates, registry presence and KV events (after the
reference's crates/kvbm-logical/src/manager/tests.rs and events/tests.rs)."""


import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from kvbm_b200 import _core_native as core
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import TokenBlockSequence, lineage, parent, position, sequence_hashes


def seq(n_blocks, start=0, bs=4, salt=None):
    return sequence_hashes(list(range(start, start + n_blocks * bs)), bs, salt)


def fill(mgr, hashes):
    blocks = mgr.allocate_blocks(len(hashes))
    assert blocks is not None
    return [mgr.register_block(b.complete(h)) for b, h in zip(blocks, hashes)]


def test_hash_structure_and_chaining():
    h = seq(5)
    assert [position(x) for x in h] == [0, 1, 2, 3, 4]
    assert parent(h[0]) == 0
    for a, b in zip(h, h[1:]):
        assert parent(b) == lineage(a)
    # same tokens, different salt -> different lineage; prefix property holds
    assert seq(5, salt="lora-a")[0] != h[0]
    assert seq(3) == h[:3]
    # incremental == batch
    s = TokenBlockSequence(list(range(6)), block_size=4)
    s.append(list(range(6, 20)))
    assert s.sequence_hashes == h[:5]
    assert list(s.partial_tokens) == []


def test_allocate_register_match_release():
    mgr = BlockManager(8, block_size=4, inactive="lru")
    assert mgr.total_blocks() == 8 and mgr.available_blocks() == 8
    h = seq(4)
    imm = fill(mgr, h)
    assert mgr.available_blocks() == 4 and mgr.active_len() == 4
    got = mgr.match_blocks(h + seq(1, start=999))
    assert [g.block_id for g in got] == [b.block_id for b in imm]
    del got, imm
    assert mgr.inactive_len() == 4 and mgr.available_blocks() == 8
    # inactive blocks are still matchable (resurrection)
    got = mgr.match_blocks(h[:2])
    assert len(got) == 2 and mgr.inactive_len() == 2
    m = mgr.metrics()
    assert m["registrations"] == 4 and m["match_blocks_returned"] == 6


def test_match_stops_at_first_miss_scan_does_not():
    mgr = BlockManager(8, block_size=4, inactive="lru")
    h = seq(4)
    keep = fill(mgr, [h[0], h[1], h[3]])
    assert len(mgr.match_blocks(h)) == 2
    found = mgr.scan_matches(h)
    assert set(found) == {h[0], h[1], h[3]}
    del keep


def test_allocate_is_all_or_nothing_and_reports_evictions():
    mgr = BlockManager(4, block_size=4, inactive="lru")
    h = seq(4)
    imm = fill(mgr, h)
    assert mgr.allocate_blocks(1) is None  # everything active
    for b in imm:
        b.release()
    blocks, evicted = mgr.allocate_blocks_with_evictions(3)
    assert evicted == h[:3]  # LRU: release order
    assert mgr.allocate_blocks(2) is None
    assert mgr.match_blocks([h[3]])[0].sequence_hash == h[3]
    del blocks


def test_lineage_evicts_leaves_first():
    mgr = BlockManager(5, block_size=4, inactive="lineage")
    trunk = seq(3)
    branch_a = sequence_hashes(list(range(12)) + [100, 101, 102, 103], 4)[3:]
    branch_b = sequence_hashes(list(range(12)) + [200, 201, 202, 203], 4)[3:]
    imm = fill(mgr, trunk + branch_a + branch_b)
    # release the trunk first: a plain LRU would evict it first
    for b in imm[:3]:
        b.release()
    for b in imm[3:]:
        b.release()
    keep, evicted = mgr.allocate_blocks_with_evictions(2)
    assert set(evicted) == {branch_a[0], branch_b[0]}
    keep2, evicted = mgr.allocate_blocks_with_evictions(3)
    assert evicted == [trunk[2], trunk[1], trunk[0]]


def test_multi_lru_keeps_hot_blocks():
    freq = core.TinyLfu(1024)
    mgr = BlockManager(4, block_size=4, inactive="multi_lru", frequency=freq)
    hot, cold = seq(1), seq(1, start=50)
    for _ in range(5):
        freq.touch(lineage(hot[0]))
    imm = fill(mgr, hot + cold)
    del imm
    _, ev = mgr.allocate_blocks_with_evictions(3)
    assert cold[0] in ev and hot[0] not in ev


def test_duplicate_policies():
    h = seq(1)
    allow = BlockManager(4, block_size=4, inactive="lru", duplicate_policy="allow")
    a = fill(allow, h)
    b = fill(allow, h)
    assert b[0].kind == "duplicate" and b[0].block_id != a[0].block_id
    assert allow.metrics()["duplicate_blocks"] == 1
    del a
    # the duplicate keeps its primary alive
    assert allow.active_len() == 1
    del b
    assert allow.inactive_len() == 1 and allow.reset_len() == 3

    rej = BlockManager(4, block_size=4, inactive="lru", duplicate_policy="reject")
    a = fill(rej, h)
    b = fill(rej, h)
    assert b[0].block_id == a[0].block_id
    assert rej.metrics()["registration_dedup"] == 1 and rej.reset_len() == 3


def test_reset_on_release_and_reset_inactive_pool():
    mgr = BlockManager(4, block_size=4, inactive="lru")
    imm = fill(mgr, seq(2))
    imm[0].set_reset_on_release(True)
    del imm
    assert mgr.inactive_len() == 1 and mgr.reset_len() == 3
    mgr.reset_inactive_pool()
    assert mgr.reset_len() == 4


def test_type_state_misuse_raises():
    mgr = BlockManager(2, block_size=4)
    b = mgr.allocate_blocks(1)[0]
    c = b.complete(seq(1)[0])
    with pytest.raises(RuntimeError):
        b.complete(seq(1)[0])
    mb = c.reset()
    with pytest.raises(RuntimeError):
        c.release() or c.reset()
    mb.release()
    assert mgr.reset_len() == 2


def test_events_create_remove_across_tiers_and_policy():
    q = core.EventQueue(all_events=True)
    reg = core.Registry(events=q)
    g2 = BlockManager(4, block_size=4, inactive="lru", tier=Tier.G2, registry=reg)
    g3 = BlockManager(4, block_size=4, inactive="lru", tier=Tier.G3, registry=reg)
    h = seq(2)
    a = fill(g2, h)
    b = fill(g3, h[:1])
    assert [k for k, _ in q.drain()] == ["create", "create"]
    assert reg.presence_mask(h[0]) == (1 << Tier.G2) | (1 << Tier.G3)
    del a
    g2.reset_inactive_pool()  # h[1] leaves the instance, h[0] is still in G3
    ev = q.drain()
    assert ev == [("remove", h[1])]
    del b
    g3.reset_inactive_pool()
    assert q.drain() == [("remove", h[0])]

    p2 = core.EventQueue(all_events=False, min_position=2, max_position=8)
    mgr = BlockManager(16, block_size=4, registry=core.Registry(events=p2))
    imm = fill(mgr, seq(10))
    created = [position(x) for _, x in p2.drain()]
    assert created == [2, 4, 8]
    del imm


def test_event_batches_are_sorted():
    q = core.EventQueue()
    mgr = BlockManager(8, block_size=4, registry=core.Registry(events=q))
    h = seq(4)
    imm = fill(mgr, h)
    del imm
    mgr.reset_inactive_pool()
    batches = q.drain_batches(3)
    kinds = [k for k, _ in batches]
    assert kinds == ["create", "create", "remove", "remove"]
    assert [position(x) for x in batches[0][1]] == [0, 1, 2]
    rem = batches[2][1] + batches[3][1]
    assert all(position(a) >= position(b) for a, b in zip(batches[2][1], batches[2][1][1:]))
    assert sorted(rem) == sorted(h)


@settings(max_examples=60, deadline=None)
@given(st.lists(st.tuples(st.sampled_from(["alloc", "register", "release", "match", "evict"]),
                          st.integers(0, 7)), max_size=80),
       st.sampled_from(["lru", "lineage", "multi_lru", "lineage_fifo"]))
def test_pool_invariants_random_ops(ops, backend):
    """Conservation: reset + inactive + held == total, for any op sequence."""
    N = 8
    mgr = BlockManager(N, block_size=4, inactive=backend)
    all_h = seq(8)
    mutable, held = [], []
    for op, x in ops:
        if op == "alloc":
            got = mgr.allocate_blocks(1 + x % 3)
            if got:
                mutable.extend(got)
        elif op == "register" and mutable:
            b = mutable.pop()
            held.append(mgr.register_block(b.complete(all_h[x])))
        elif op == "release" and held:
            held.pop(x % len(held)).release()
        elif op == "match":
            held.extend(mgr.match_blocks(all_h[: x + 1]))
        elif op == "evict":
            got = mgr.allocate_blocks(1)
            if got:
                got[0].release()
        primaries = {b.block_id for b in held}
        assert mgr.reset_len() + mgr.inactive_len() + len(mutable) + len(primaries) <= N
        assert mgr.available_blocks() == mgr.reset_len() + mgr.inactive_len()
    for b in mutable + held:
        b.release()
    assert mgr.available_blocks() == N


def test_positional_index_deepest_holder():
    ix = core.PositionalIndex(1024, 4)
    h = seq(6)
    ix.apply(7, "create", h[:4])
    ix.apply(9, "create", h[:2])
    deepest, holders = ix.query_holders(h)
    assert deepest == h[3] and holders == [7]
    ix.remove_instance(7)
    deepest, holders = ix.query_holders(h)
    assert deepest == h[1] and holders == [9]
    ix.apply(9, "remove", h[:2])
    assert ix.query_holders(h) is None
    small = core.PositionalIndex(8, 4)
    small.apply(1, "create", h)
    assert small.dropped_out_of_range() == 4


def test_consolidator_first_store_last_remove():
    t = core.ConsolidatorTracker()
    toks = list(range(16))
    assert t.handle_store(0, "a", None, toks, 16)
    assert not t.handle_store(1, "x", None, toks, 16)  # same block from a second source
    assert not t.handle_store(0, "a", None, toks, 16)  # idempotent repeat
    ev = t.drain_events()
    assert [e["kind"] for e in ev] == ["store"]
    assert not t.handle_remove(0, "a")
    assert t.handle_remove(1, "x")
    assert [e["kind"] for e in t.drain_events()] == ["remove"]
    # parent resolution through external hashes
    t.handle_store(0, "p", None, toks, 16)
    t.handle_store(0, "c", "p", list(range(16, 32)), 16)
    evs = t.drain_events()
    assert position(evs[1]["seq_hash"]) == 1 and parent(evs[1]["seq_hash"]) == lineage(evs[0]["seq_hash"])
    # KVBM-only blocks are not publishable until a token-carrying source arrives
    h = seq(1, start=500)[0]
    assert t.handle_kvbm_store(h)
    assert t.drain_events() == []
    t.handle_clear_all()
    assert t.drain_events()[-1]["kind"] == "clear_all" and t.num_blocks() == 0


@settings(max_examples=50, deadline=None)
@given(st.lists(st.tuples(st.sampled_from(["store", "remove", "clear"]), st.integers(0, 2), st.integers(0, 5)),
                max_size=60))
def test_consolidator_chaos_invariants(ops):
    """STORE is published only for a block not live downstream, REMOVE only for a live one."""
    t = core.ConsolidatorTracker()
    live = set()
    for op, src, blk in ops:
        if op == "store":
            t.handle_store(src, f"b{blk}", None, [blk] * 4, 4)
        elif op == "remove":
            t.handle_remove(src, f"b{blk}")
        else:
            t.handle_clear_all()
        for e in t.drain_events():
            if e["kind"] == "store":
                assert e["seq_hash"] not in live
                live.add(e["seq_hash"])
            elif e["kind"] == "remove":
                assert e["seq_hash"] in live
                live.remove(e["seq_hash"])
            else:
                live.clear()


def test_tinylfu_counts_and_ages():
    f = core.TinyLfu(64)
    for _ in range(7):
        f.touch(42)
    assert f.estimate(42) >= 7
    assert f.estimate(43) <= 1
    for i in range(2000):
        f.touch(1000 + i)
    assert f.estimate(42) < 7  # halved by ageing


def test_lock_hierarchy_is_checked():
    assert core.lock_check_enabled()  # turned on for the whole test run
    with pytest.raises(core.LockOrderError, match="Registry .* while holding BlockPool"):
        core.lock_order_selftest()
    # a full allocate / register / match / release cycle respects the hierarchy
    mgr = BlockManager(8, 16, "multi_lru", Tier.G2)
    blocks = mgr.allocate_blocks(2)
    imm = mgr.register_mutable(blocks, sequence_hashes(list(range(32)), 16))
    assert len(mgr.match_blocks([b.sequence_hash for b in imm])) == 2


def test_pool_micro_benchmark_runs():
    from kvbm_b200.bench.pool_bench import micro

    out = micro(n=64, reps=3)
    for api in ("native_batch_ns_per_block", "handles_ns_per_block"):
        assert set(out[api]) == {"match_active", "match_inactive", "drop"}
        assert all(v > 0 for v in out[api].values())


def test_register_mutable_released_caches_without_handles():
    from kvbm_b200.logical.manager import BlockManager, Tier
    from kvbm_b200.logical.sequence import sequence_hashes

    m = BlockManager(8, 16, "lru", Tier.G2)
    hs = sequence_hashes(list(range(4 * 16)), 16)
    blocks = m.allocate_blocks(4)
    assert m.register_mutable_released(blocks, hs) == 4
    assert m.inactive_len() == 4 and m.count_prefix(hs) == 4
    got = m.match_blocks(hs)
    assert [b.sequence_hash for b in got] == hs
    for b in got:
        b.release()
    assert m.allocate_blocks_with_evictions(8) is not None  # four free + four evictable
