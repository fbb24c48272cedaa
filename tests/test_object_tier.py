"""CPU tests of the G4 tier: G2 -> G4 offload executor and G4 -> G2 staging on a find."""

import torch

from kvbm_b200.engine.leader import InstanceLeader, ParallelWorkers
from kvbm_b200.engine.object_tier import ObjectTier
from kvbm_b200.engine.offload import OffloadItem, OffloadPipeline, make_policy
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.object.store import FsObjectStore
from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
from kvbm_b200.physical.verify import FillPattern, checksum_blocks, fill_blocks


def _g2(nb=12, ranks=2):
    cfg = LayoutConfig.for_model(nb, 2, 2, 64, 16)
    out = []
    for _ in range(ranks):
        n = KvLayout._strides(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, True)[-1]
        out.append(KvLayout.over_tensor(cfg, torch.zeros(n, dtype=torch.uint8)))
    return out


def test_offload_to_g4_and_stage_back_per_rank(tmp_path):
    store = FsObjectStore(str(tmp_path))
    src_layouts = _g2()
    tier = ObjectTier(store, src_layouts)
    hs = sequence_hashes(list(range(16 * 5)), 16)
    for r, lay in enumerate(src_layouts):
        fill_blocks(lay, [0, 1, 2, 3], FillPattern.RANDOM, seed=r)
    want = [checksum_blocks(lay, [0, 1, 2]) for lay in src_layouts]

    # G2 -> G4 through an offload pipeline with the object-presence policy
    p = OffloadPipeline("g2_to_g4", None, tier.executor(), make_policy(["object_presence"], None, store))
    h = p.enqueue([OffloadItem(x, i) for i, x in enumerate(hs[:3])])
    assert h.wait(10).value == "done" and tier.stats["put_blocks"] == 3
    h2 = p.enqueue([OffloadItem(x, i) for i, x in enumerate(hs[:3])])
    assert h2.wait(10).value == "done" and len(h2.skipped) == 3  # already in G4
    p.close()
    assert store.has(store.key(hs[0], rank=1))

    # another instance (fresh G2) finds the prefix in G4
    dst_layouts = _g2()
    g2 = BlockManager(12, 16, "lru", Tier.G2)
    leader = InstanceLeader(g2, ParallelWorkers([]), object_store=ObjectTier(store, dst_layouts))
    res = leader.find_matches(hs)
    assert res.num_blocks == 3 and res.staged_from_g4 == 3
    ids = [b.block_id for b in res.g2_blocks]
    assert [checksum_blocks(lay, ids) for lay in dst_layouts] == want
    res.release()
    # now they are plain G2 hits
    res2 = leader.find_matches(hs)
    assert res2.num_blocks == 3 and getattr(res2, "staged_from_g4", 0) == 0
    res2.release()
    store.close()
