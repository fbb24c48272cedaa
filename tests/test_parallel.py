"""Heterogeneous-TP planning and P2P session protocol (CPU)."""

import threading
import time

import pytest

from kvbm_b200.parallel.session import Lifecycle, SessionError, SessionManager
from kvbm_b200.parallel.tp import CompatError, ParallelismTemplate, Shard, plan_pull, plan_push, validate


def T(tp, heads=8, layers=80):
    return ParallelismTemplate(tp_size=tp, global_heads=heads, num_layers=layers)


def test_plan_symmetric():
    plans = plan_pull(T(2), T(2))
    assert [p.shards for p in plans] == [[Shard(0, 0, 0, 4)], [Shard(1, 0, 0, 4)]]


def test_plan_local_smaller_pulls_from_many():
    # decode TP=2 pulling from prefill TP=4: each decode rank assembles 4 heads from 2 ranks
    plans = plan_pull(T(2), T(4))
    assert plans[0].shards == [Shard(0, 0, 0, 2), Shard(1, 0, 2, 2)]
    assert plans[1].shards == [Shard(2, 0, 0, 2), Shard(3, 0, 2, 2)]


def test_plan_local_larger_takes_a_slice():
    plans = plan_pull(T(8), T(2))
    assert plans[5].shards == [Shard(1, 1 * 1, 0, 1)] or plans[5].shards == [Shard(1, 1, 0, 1)]
    assert all(len(p.shards) == 1 for p in plans)
    heads = sorted((s.remote_rank, s.remote_head_offset) for p in plans for s in p.shards)
    assert heads == [(r, o) for r in range(2) for o in range(4)]


def test_push_plan_covers_every_head_once():
    for src_tp, dst_tp in [(4, 2), (2, 4), (1, 8), (8, 1), (2, 2)]:
        push = plan_push(T(src_tp), T(dst_tp))
        covered = set()
        for src, targets in enumerate(push):
            for t in targets:
                for h in range(t.num_heads):
                    g_src = src * (8 // src_tp) + t.src_head_offset + h
                    g_dst = t.dst_rank * (8 // dst_tp) + t.dst_head_offset + h
                    assert g_src == g_dst
                    covered.add(g_dst)
        assert covered == set(range(8))


@pytest.mark.parametrize("a,b", [(T(3, heads=6), T(2, heads=6)), (T(2), T(2, layers=32)),
                                 (ParallelismTemplate(2, 8, 80, pp_size=2), T(2)),
                                 (T(2), ParallelismTemplate(2, 8, 80, shard_axis="layer"))])
def test_incompatible_templates_rejected(a, b):
    with pytest.raises(CompatError):
        validate(a, b)


def test_session_commit_available_stream():
    mgr = SessionManager(attach_timeout=5)
    s = mgr.open(initiator=1, holder=2)
    got = []

    def puller():
        s.wait_attached(5)
        while True:
            new = s.drain_available(timeout=5)
            got.extend(new)
            if not new:
                break

    t = threading.Thread(target=puller)
    t.start()
    s.attach()
    s.commit([10, 11, 12])
    with pytest.raises(SessionError):
        s.make_available([99])  # not committed
    s.make_available([10])
    s.make_available([11, 12])
    s.finish_commits()
    s.finish_availability()
    t.join(5)
    assert got == [10, 11, 12] and s.lifecycle == Lifecycle.DRAINED
    mgr.close()


def test_session_rules_and_watchdog():
    mgr = SessionManager(attach_timeout=0.1, sweep_s=0.02)
    s = mgr.open(1, 2)
    s.commit([1])
    with pytest.raises(SessionError):
        s.finish_availability()  # commits still open
    s.finish_commits()
    with pytest.raises(SessionError):
        s.finish_availability()  # committed block never available
    time.sleep(0.3)
    assert len(mgr) == 0 and s.lifecycle == Lifecycle.FAILED
    with pytest.raises(SessionError):
        s.drain_available(timeout=0.1)
    mgr.close()
