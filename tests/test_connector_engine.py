"""CPU tests of the connector <-> engine seam (LeaderEngine)."""

import concurrent.futures as cf

import pytest

from kvbm_b200.connector.engine import LocalConnectorEngine, NoopBlockEngine, Status
from kvbm_b200.engine.leader import InstanceLeader, ParallelWorkers
from kvbm_b200.engine.offload import OffloadEngine, OffloadPipeline, PresenceFilter
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.physical.transfer import TransferCompleteNotification


class _Worker:
    def __init__(self):
        self.copies = []

    def execute_local_transfer(self, src_tier, src_ids, dst_tier, dst_ids, layer_range=None):
        self.copies.append((src_tier, list(src_ids), dst_tier, list(dst_ids)))
        return TransferCompleteNotification.ready()


def _leader(nb=16):
    g2 = BlockManager(nb, 16, "lru", Tier.G2)
    w = _Worker()
    return InstanceLeader(g2, ParallelWorkers([w])), g2, w


def _cache(g2, hashes):
    blocks = g2.allocate_blocks(len(hashes))
    for b in g2.register_mutable(blocks, hashes):
        b.release()


def test_noop_engine():
    e = NoopBlockEngine()
    h = e.find_blocks("r", sequence_hashes(list(range(64)), 16))
    assert h.status == Status.READY and h.num_blocks == 0
    assert e.onboard_blocks("r", h.search_id, []) == 0 and e.poll_action(0) == Status.DONE
    with pytest.raises(ValueError):
        e.onboard_blocks("r", h.search_id, [1])
    assert e.take_offload_drain() == [] and e.evict("r") == 0


def test_local_find_onboard_release():
    leader, g2, w = _leader()
    hs = sequence_hashes(list(range(16 * 5)), 16)
    _cache(g2, hs[:3])
    e = LocalConnectorEngine(leader)
    h = e.find_blocks("r", hs)
    assert h.status == Status.READY and h.num_blocks == 3
    aid = e.onboard_blocks("r", h.search_id, [7, 8])  # the third match is released
    assert e.poll_action(aid) == Status.DONE
    assert w.copies and w.copies[0][3] == [7, 8]
    e.release_action(aid)
    e.release_search(h.search_id)
    assert e.poll_action(aid) == Status.RELEASED
    assert g2.allocate_blocks(16) is not None  # every reference was dropped


def test_local_remote_search_stalls_until_the_pull_lands():
    leader, g2, _ = _leader()
    hs = sequence_hashes(list(range(16 * 4)), 16)
    _cache(g2, hs[:1])
    fut = cf.Future()

    class _Remote:
        def start(self, missing):
            assert missing == hs[1:]
            return fut

    e = LocalConnectorEngine(leader, remote_search=_Remote())
    h = e.find_blocks("r", hs)
    assert e.poll_search(h.search_id).status == Status.PENDING
    _cache(g2, hs[1:3])  # what the pull registers
    fut.set_result(2)
    h = e.poll_search(h.search_id)
    assert h.status == Status.READY and h.num_blocks == 3
    e.release_search(h.search_id)
    with pytest.raises(KeyError):
        e.poll_search(h.search_id)


def test_offload_buffer_flushes_after_the_pass_and_evicts():
    leader, g2, _ = _leader()
    eng = OffloadEngine()

    def executor(items):
        blocks = g2.allocate_blocks(len(items))
        return g2.register_mutable(blocks, [i.seq_hash for i in items])

    eng.add(OffloadPipeline("g1_to_g2", g2, executor, PresenceFilter(g2)))
    leader.offload_engine = eng
    e = LocalConnectorEngine(leader)
    hs = sequence_hashes(list(range(16 * 6)), 16)
    e.offload("a", hs[:2], [0, 1])
    e.offload("b", hs[2:4], [2, 3])
    assert e.evict("b") == 1
    drained = e.take_offload_drain()
    assert [r for r, _ in drained] == ["a"]
    assert drained[0][1].wait(5).value == "done"
    assert len(g2.match_blocks(hs[:2])) == 2
    eng.close()
