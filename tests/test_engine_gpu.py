"""Tier transfers through the TransferManager, offload pipelines and the
InstanceLeader on one GPU (G1 device, G2 pinned host, G3 local disk)."""


import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.engine.leader import InstanceLeader, ParallelWorkers, StagingMode, FindMatchesOptions
from kvbm_b200.engine.offload import (OffloadEngine, OffloadItem, OffloadPipeline, PresenceFilter,
                                      make_tier_executor)
from kvbm_b200.engine.worker import Worker
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig

NHD = KvBlockLayout.OPERATIONAL_NHD


def _bits(t):
    """Bitwise view: random bytes contain NaN patterns, so compare raw bits."""
    return t.contiguous().view(torch.int16)


def _g1(nb=32, kind="layer_separate"):
    cfg = LayoutConfig.for_model(nb, 4, 8, 128, 16)
    g1 = KvLayout.allocate(cfg, kind, NHD)
    g1._flat().random_(0, 256)
    return g1


@pytest.mark.parametrize("engine", ["auto", "tile", "ce"])
def test_tier_roundtrip_g1_g2_g3(engine, tmp_path):
    g1 = _g1(kind="fully_contiguous")
    w = Worker(0, g1, g2_blocks=16, g3_blocks=16, g3_path=str(tmp_path / "g3.bin"), engine=engine)
    src = [3, 9, 1, 30]
    ref = g1.gather_blocks(src).clone()
    w.execute_local_transfer(Tier.G1, src, Tier.G2, [0, 1, 2, 3]).wait()
    w.execute_local_transfer(Tier.G2, [0, 1, 2, 3], Tier.G3, [5, 6, 7, 8]).wait()
    # G3 -> G1 goes through the pinned bounce buffer (two hops)
    w.execute_local_transfer(Tier.G3, [5, 6, 7, 8], Tier.G1, [10, 11, 12, 13]).wait()
    torch.cuda.synchronize()
    assert torch.equal(_bits(g1.gather_blocks([10, 11, 12, 13])), _bits(ref))
    # G1 -> G3 directly (two hops)
    w.execute_local_transfer(Tier.G1, [10, 11], Tier.G3, [0, 1]).wait()
    w.execute_local_transfer(Tier.G3, [0, 1], Tier.G2, [14, 15]).wait()
    assert torch.equal(_bits(w.g2_layout.gather_blocks([14, 15]).cuda()), _bits(ref[:2]))
    with pytest.raises(IndexError):
        w.execute_local_transfer(Tier.G1, [99], Tier.G2, [0])
    w.close()


def test_two_hop_larger_than_the_bounce(tmp_path):
    # 10 blocks through a 4-block bounce: three chunks each way
    g1 = _g1(kind="fully_contiguous")
    w = Worker(0, g1, g2_blocks=4, g3_blocks=16, g3_path=str(tmp_path / "g3.bin"), bounce_blocks=4)
    src, slots, dst = list(range(2, 12)), list(range(3, 13)), list(range(20, 30))
    ref = g1.gather_blocks(src).clone()
    w.execute_local_transfer(Tier.G1, src, Tier.G3, slots).wait()
    w.execute_local_transfer(Tier.G3, slots, Tier.G1, dst).wait()
    torch.cuda.synchronize()
    assert torch.equal(_bits(g1.gather_blocks(dst)), _bits(ref))
    w.close()


def test_layer_selection_and_layerwise_onboard():
    g1 = _g1()
    w = Worker(0, g1, g2_blocks=8)
    ref = g1.gather_blocks([4, 5]).clone()
    w.tm.execute_transfer_selection(w.handles.g1, [4, 5], w.handles.g2, [0, 1], layer_range=(1, 3)).wait()
    got = w.g2_layout.gather_blocks([0, 1]).cuda()
    assert torch.equal(_bits(got[:, 1:3]), _bits(ref[:, 1:3]))
    w.execute_local_transfer(Tier.G1, [4, 5], Tier.G2, [0, 1]).wait()
    w.start_layerwise_onboard([0, 1], [20, 21])
    s = torch.cuda.Stream()
    for l in range(4):
        w.wait_for_layer_load(l, s)
    s.synchronize()
    assert torch.equal(_bits(g1.gather_blocks([20, 21])), _bits(ref))


def test_offload_pipeline_and_leader_find_onboard(tmp_path):
    g1 = _g1()
    w = Worker(0, g1, g2_blocks=16, g3_blocks=16, g3_path=str(tmp_path / "g3.bin"))
    g2 = BlockManager(16, 16, "lineage", Tier.G2)
    g3 = BlockManager(16, 16, "lineage", Tier.G3, registry=g2.registry)
    eng = OffloadEngine()
    p23 = OffloadPipeline("g2_to_g3", g3, make_tier_executor(w.handles.g2, g3, w.handles.g3, w.tm),
                          PresenceFilter(g3))
    chain = lambda blocks: p23.enqueue([OffloadItem(b.sequence_hash, b.block_id, b.clone()) for b in blocks])
    p12 = OffloadPipeline("g1_to_g2", g2, make_tier_executor(w.handles.g1, g2, w.handles.g2, w.tm),
                          PresenceFilter(g2), on_registered=chain)
    eng.add(p12)
    eng.add(p23)
    leader = InstanceLeader(g2, ParallelWorkers([w]), g3=g3, offload=eng)
    hashes = sequence_hashes(list(range(80)), 16)
    ref = g1.gather_blocks([0, 1, 2, 3, 4]).clone()
    ev = torch.cuda.Event()
    ev.record()
    h = leader.offload_g1(hashes, [0, 1, 2, 3, 4], precondition=ev.query)
    assert h.wait(30).value == "done"
    # duplicate offload is filtered by presence
    h2 = leader.offload_g1(hashes, [0, 1, 2, 3, 4])
    assert h2.wait(30).value == "done" and len(h2.skipped) == 5
    import time
    t0 = time.time()
    while g3.inactive_len() < 5 and time.time() - t0 < 30:
        time.sleep(0.05)
    assert g3.inactive_len() == 5
    # drop G2: a find must stage from G3
    g2.reset_inactive_pool()
    res = leader.find_matches(hashes, FindMatchesOptions(staging=StagingMode.FULL))
    assert res.staged_from_g3 == 5 and len(res.g2_blocks) == 5
    note = leader.onboard(res.g2_blocks, [10, 11, 12, 13, 14])
    note.wait()
    torch.cuda.synchronize()
    assert torch.equal(_bits(g1.gather_blocks([10, 11, 12, 13, 14])), _bits(ref))
    res.release()
    eng.close()
    w.close()
