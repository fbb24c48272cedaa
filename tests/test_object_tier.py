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


def test_connector_chains_g2_to_g4_and_fetches_g4_hits_through_its_workers(tmp_path):
    """The connector path: registered G2 blocks are uploaded by the workers (store ops), and after
    G2 lost them a new request's prefix is found in G4, fetched by the workers into fresh G2 blocks
    ahead of the onboard (fetch op) and registered in G2 once the onboard is reported."""
    from kvbm_b200.connector.leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
    from kvbm_b200.connector.protocol import ConnectorMetadata

    store = FsObjectStore(str(tmp_path))
    [g2_pool] = _g2(nb=8, ranks=1)                       # the worker's G2 pool
    worker_tier = ObjectTier(store, [g2_pool], rank_base=0)
    g2 = BlockManager(8, 16, "lru", Tier.G2)
    L = ConnectorLeader(InstanceLeader.scheduler_side(g2), 16, objects=store)

    def step(n, sched, reports=None):
        m = ConnectorMetadata.decode(L.build_connector_meta(SchedulerOutputLite(n, sched)))
        for op in m.store:                               # what the worker's upload thread does
            worker_tier.put(op.hashes, op.g2_ids)
        for op in m.fetch:                               # what the worker does before the onboards
            assert all(worker_tier.get_into(op.hashes, op.g2_ids))
        rep = dict(reports or {})
        if m.store:
            rep["stored"] = {m.step: 1}
        L.update_connector_output(finished_sending=set(), finished_recving=set(), worker_meta=rep or None)
        return m

    tokens = list(range(5 * 16 + 3))
    hs = sequence_hashes(tokens, 16)
    L.create_slot(KvbmRequest("a", tokens))
    assert L.get_num_new_matched_tokens("a", 0) == (0, False)
    L.update_state_after_alloc("a", [0, 1, 2, 3, 4, 5], 0)
    m = step(1, {"a": ([], [], len(tokens))})
    [off] = m.offload
    fill_blocks(g2_pool, off.g2_ids, FillPattern.RANDOM, seed=5)  # the worker's G1 -> G2 copy
    want = checksum_blocks(g2_pool, off.g2_ids)
    L.update_connector_output(finished_sending={"a"}, finished_recving=set(), worker_meta={"offloaded": {1: 1}})
    L.request_finished("a")
    m2 = step(2, {})                                     # the registered G2 blocks chain to G4
    assert [len(op.g2_ids) for op in m2.store] == [5]
    assert all(store.has(store.key(h, rank=0)) for h in hs[:5])
    assert L.engine.stats["stored_to_g4"] == 5
    g2.reset_inactive_pool()                             # G2 forgets them (evicted)
    g2_pool.backing.zero_()
    assert g2.count_prefix(hs) == 0

    L.create_slot(KvbmRequest("b", tokens))
    assert L.get_num_new_matched_tokens("b", 0) == (5 * 16, True)  # all five from G4
    L.update_state_after_alloc("b", [10, 11, 12, 13, 14, 15], 5 * 16)
    m3 = step(3, {"b": ([], [], 5 * 16)})
    [f] = m3.fetch
    [on] = m3.onboard
    assert f.hashes == hs[:5] and on.g2_ids == f.g2_ids and on.g1_ids == [10, 11, 12, 13, 14]
    assert checksum_blocks(g2_pool, f.g2_ids) == want   # the bytes came back from the store
    L.update_connector_output(finished_sending=set(), finished_recving={"b"}, worker_meta=None)
    assert g2.count_prefix(hs) == 5 and L.engine.stats["staged_from_g4"] == 5
    store.close()


def test_worker_fetch_of_a_missing_object_reports_load_errors(tmp_path):
    """A G4 object that vanished between the leader's presence check and the worker's fetch: the
    G1 blocks it would have filled are reported as load errors (the framework recomputes them)."""
    from kvbm_b200.connector.protocol import ConnectorMetadata, FetchOp, OnboardOp
    from kvbm_b200.connector.worker import ConnectorWorker

    store = FsObjectStore(str(tmp_path))
    [g2_pool] = _g2(nb=8, ranks=1)
    tier = ObjectTier(store, [g2_pool])
    hs = sequence_hashes(list(range(3 * 16)), 16)
    tier.put(hs[:2], [0, 1])                      # the third object is missing
    w = ConnectorWorker(device=0)
    w.objects = tier
    meta = ConnectorMetadata(step=1, onboard=[OnboardOp("r", [4, 5, 6], [20, 21, 22])],
                             fetch=[FetchOp("r", hs, [4, 5, 6])])
    w._fetch(meta.fetch[0], meta)
    assert w.get_block_ids_with_load_errors() == {22}
    store.close()
