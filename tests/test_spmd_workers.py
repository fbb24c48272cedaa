"""Tensor-parallel worker group across processes, on CPU: the leader fans
every block operation out to each rank's worker service over the messenger
(each rank moves its own head shard) and the operation completes when every
rank's part does; a failing rank fails the operation."""

import multiprocessing as mp
import time

import pytest

from kvbm_b200.engine.leader import FindMatchesOptions, InstanceLeader, StagingMode
from kvbm_b200.engine.spmd import SpmdParallelWorkers
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.physical.transfer import TransferCompleteNotification
from kvbm_b200.runtime.messenger import Messenger


class _Cfg:
    num_heads, num_layers, bytes_per_block = 4, 2, 4096


class _Layout:
    config = _Cfg()


class FakeWorker:
    """Records the ops a rank is asked to run; ``fail`` makes every transfer raise."""

    def __init__(self, fail=False):
        self.ops, self.fail, self.g1_layout = [], fail, _Layout()

    def execute_local_transfer(self, src, src_ids, dst, dst_ids, layer_range=None):
        if self.fail:
            raise RuntimeError("rank failed")
        self.ops.append((int(src), list(src_ids), int(dst), list(dst_ids), layer_range))
        return TransferCompleteNotification.ready()

    def start_layerwise_onboard(self, g2_ids, g1_ids):
        self.ops.append(("layerwise", list(g2_ids), list(g1_ids)))


def _rank_main(rank, fail, q, stop):
    from kvbm_b200.engine.spmd import WorkerService

    m = Messenger(bind="tcp://127.0.0.1:0")
    w = FakeWorker(fail=fail)
    WorkerService(m, w, rank)
    m.register_handler("test.ops", lambda _p: [list(map(lambda x: list(x) if isinstance(x, (list, tuple)) else x, op))
                                               for op in w.ops])
    q.put((rank, m.instance_id, m.address))
    stop.wait(60)
    m.close()


def _group(n, fail_rank=None):
    ctx = mp.get_context("spawn")
    q, stop = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_rank_main, args=(r, r == fail_rank, q, stop), daemon=True) for r in range(n)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=60) for _ in range(n))
    leader_m = Messenger(bind="tcp://127.0.0.1:0")
    for _, iid, addr in got:
        leader_m.register_peer(iid, addr)
    return leader_m, [iid for _, iid, _ in got], procs, stop


def test_every_rank_runs_the_same_block_op_and_completion_aggregates():
    m, iids, procs, stop = _group(2)
    try:
        group = SpmdParallelWorkers(m, iids, timeout=20)
        assert [l["rank"] for l in group.layouts()] == [0, 1]
        g2 = BlockManager(16, 16, "lru", Tier.G2)
        g3 = BlockManager(16, 16, "lru", Tier.G3, registry=g2.registry)
        leader = InstanceLeader(g2, group, g3=g3)
        # put 3 blocks in G3, then find them with full staging: the leader stages through both ranks
        hashes = [11, 22, 33]
        dst, _ = g3.allocate_blocks_with_evictions(3)
        for b in g3.register_mutable(dst, hashes):
            b.release()
        res = leader.find_matches(hashes, FindMatchesOptions(staging=StagingMode.FULL))
        assert len(res.g2_blocks) == 3 and res.staged_from_g3 == 3
        note = group.execute_local_transfer(Tier.G2, [0, 1], Tier.G1, [5, 6], layer_range=(0, 1))
        note.wait(timeout=20)
        assert note.is_complete()
        ops = [m.call(iid, "test.ops", None) for iid in iids]
        assert ops[0] == ops[1] and len(ops[0]) == 2
        assert ops[0][0][0] == int(Tier.G3) and ops[0][0][2] == int(Tier.G2)
        assert ops[0][1] == [int(Tier.G2), [0, 1], int(Tier.G1), [5, 6], [0, 1]]
        res.release()
        group.close()
    finally:
        stop.set()
        for p in procs:
            p.join(timeout=10)
        m.close()


def test_a_failing_rank_fails_the_op():
    m, iids, procs, stop = _group(2, fail_rank=1)
    try:
        group = SpmdParallelWorkers(m, iids, timeout=20)
        note = group.execute_local_transfer(Tier.G2, [0], Tier.G1, [1])
        t0 = time.monotonic()
        with pytest.raises(Exception):
            note.wait(timeout=20)
        assert time.monotonic() - t0 < 20
        group.close()
    finally:
        stop.set()
        for p in procs:
            p.join(timeout=10)
        m.close()
