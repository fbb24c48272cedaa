"""Connector leader logic on CPU (no GPU): matching, onboard planning,
save-cursor offloads, delayed frees; and the step-metadata wire format."""


import pytest

from kvbm_b200.connector.leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
from kvbm_b200.connector.protocol import (ConnectorMetadata, OffloadOp, OnboardOp, PushOp, RecvOp, SpillOp,
                                          StageOp)
from kvbm_b200.engine.leader import InstanceLeader
from kvbm_b200.logical.manager import BlockManager, Tier


def make_leader(g2_blocks=64, bs=16):
    g2 = BlockManager(g2_blocks, bs, "lineage", Tier.G2)
    return ConnectorLeader(InstanceLeader.scheduler_side(g2), bs)


def step(leader, n, sched):
    return ConnectorMetadata.decode(leader.build_connector_meta(SchedulerOutputLite(n, sched)))


def test_cold_request_offloads_complete_blocks():
    L = make_leader()
    prompt = list(range(100))
    L.create_slot(KvbmRequest("a", prompt))
    assert L.get_num_new_matched_tokens("a", 0) == (0, False)
    L.update_state_after_alloc("a", list(range(7)), 0)
    # chunked prefill: 48 tokens, then the rest
    m = step(L, 1, {"a": ([], [], 48)})
    assert [o.g1_ids for o in m.offload] == [[0, 1, 2]] and not m.onboard
    m = step(L, 2, {"a": ([], [], 100)})
    assert m.offload[0].g1_ids == [3, 4, 5]  # 100 tokens -> 6 complete blocks
    assert L.request_finished("a") == (True, None)  # offload still in flight
    L.update_connector_output(finished_sending={"a"})
    assert L.num_slots() == 0


def test_warm_request_onboards_and_skips_present_blocks():
    L = make_leader()
    prompt = list(range(100))
    L.create_slot(KvbmRequest("a", prompt))
    L.get_num_new_matched_tokens("a", 0)
    L.update_state_after_alloc("a", list(range(7)), 0)
    step(L, 1, {"a": ([], [], 100)})
    L.update_connector_output(finished_sending={"a"}, worker_meta={"offloaded": {1: 1}})
    L.request_finished("a")
    # same prompt again: 6 cached blocks, but the last prompt token must be computed -> 6 blocks (96 < 99)
    L.create_slot(KvbmRequest("b", prompt))
    n, is_async = L.get_num_new_matched_tokens("b", 0)
    assert (n, is_async) == (96, True)
    L.update_state_after_alloc("b", list(range(20, 27)), n)
    m = step(L, 2, {"b": ([], [], 100)})
    assert len(m.onboard) == 1 and m.onboard[0].g1_ids == list(range(20, 26))
    assert m.offload == []  # everything already in G2
    L.update_connector_output(finished_recving={"b"})
    assert L.request_finished("b") == (False, None)


def test_framework_prefix_hit_is_skipped():
    L = make_leader()
    prompt = list(range(64))
    L.create_slot(KvbmRequest("a", prompt))
    L.update_state_after_alloc("a", list(range(4)), 0)
    step(L, 1, {"a": ([], [], 64)})
    L.update_connector_output(worker_meta={"offloaded": {1: 1}})
    L.create_slot(KvbmRequest("b", prompt + list(range(1000, 1040))))
    # the framework already has 32 tokens in G1: KVBM contributes blocks 2..3
    n, _ = L.get_num_new_matched_tokens("b", 32)
    assert n == 32


def test_salt_separates_caches():
    L = make_leader()
    prompt = list(range(64))
    L.create_slot(KvbmRequest("a", prompt, lora_name="x"))
    L.update_state_after_alloc("a", list(range(4)), 0)
    step(L, 1, {"a": ([], [], 64)})
    L.create_slot(KvbmRequest("b", prompt, lora_name="y"))
    assert L.get_num_new_matched_tokens("b", 0) == (0, False)


def test_decode_tokens_extend_sequence_when_enabled():
    L = make_leader()
    L.decode_offload = True
    L.create_slot(KvbmRequest("a", list(range(30))))
    L.update_state_after_alloc("a", [0, 1, 2], 0)
    m = step(L, 1, {"a": ([], [], 30)})
    assert [o.g1_ids for o in m.offload] == [[0]]
    m = step(L, 2, {"a": ([7, 8], [], 32)})
    assert [o.g1_ids for o in m.offload] == [[1]]


def test_offloaded_blocks_match_only_after_every_worker_reports_the_copy():
    g2 = BlockManager(64, 16, "lineage", Tier.G2)
    L = ConnectorLeader(InstanceLeader.scheduler_side(g2), 16, num_workers=2)
    prompt = list(range(64))
    L.create_slot(KvbmRequest("a", prompt))
    L.update_state_after_alloc("a", list(range(4)), 0)
    m = step(L, 1, {"a": ([], [], 64)})
    assert [o.g1_ids for o in m.offload] == [[0, 1, 2, 3]]
    probe = prompt + [7]
    # copies still in flight: another request must not match the G2 destinations
    L.create_slot(KvbmRequest("b", probe))
    assert L.get_num_new_matched_tokens("b", 0) == (0, False)
    # the same blocks are not offloaded twice while the first copy is pending
    L.create_slot(KvbmRequest("c", prompt))
    L.update_state_after_alloc("c", list(range(10, 14)), 0)
    assert step(L, 2, {"c": ([], [], 64)}).offload == []
    L.update_connector_output(worker_meta={"offloaded": {1: 1}})  # one of two workers
    L.create_slot(KvbmRequest("d", probe))
    assert L.get_num_new_matched_tokens("d", 0) == (0, False)
    L.update_connector_output(worker_meta={"offloaded": {1: 1}})  # the second one
    L.create_slot(KvbmRequest("e", probe))
    assert L.get_num_new_matched_tokens("e", 0) == (64, True)


def test_metadata_roundtrip():
    m = ConnectorMetadata(3, [OnboardOp("r", [1, 2], [5, 6])], [OffloadOp("q", [7], [9])], ["z"],
                          stage=[StageOp("r", [4], [8])], spill=[SpillOp([3], [11])],
                          push=[PushOp("p", 7, [1, 2], [3, 4], 5, 9, True)], recv=[RecvOp("q", 2, 9, [3, 4], 1.5)])
    d = ConnectorMetadata.decode(m.encode())
    assert d == m


def test_lazy_import_does_not_pull_vllm():
    import subprocess
    import sys

    code = ("import sys; import kvbm_b200.connector.vllm_connector as m; "
            "print('vllm' in sys.modules)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "False"
    # every module of the reference package's import paths, the same way
    mods = ["kvbm", "kvbm._core", "kvbm.hub", "kvbm.hub.detect", "kvbm.hub.dispatch_lambda",
            "kvbm.hub.calibrate_lambda", "kvbm.vllm", "kvbm.vllm.config", "kvbm.vllm.consolidator_config",
            "kvbm.vllm.sched_output", "kvbm.vllm.version_check", "kvbm.vllm.dim_probe", "kvbm.vllm.connector",
            "kvbm.vllm.connector.base", "kvbm.vllm.connector.leader", "kvbm.vllm.connector.worker",
            "kvbm.vllm.connector.pd", "kvbm.vllm.connector.protocols"]
    mods += ["kvbm.kernels"]
    code = (f"import sys, importlib; [importlib.import_module(m) for m in {mods!r}]; "
            "from kvbm import KvbmRuntime, ConnectorLeader, ConnectorWorker, KvbmRequest, KvbmVllmConfig, "
            "SchedulerOutput, Tensor, kernels, _KERNELS_AVAILABLE; from kvbm.vllm import KvbmVllmConfig, "
            "version_check; from kvbm.hub import CompletionEvent, PrefillRouterHandler, try_wrap_engine, "
            "make_dispatch_lambda, make_calibrate_lambda, capture_calibration_defaults; "
            "print('vllm' in sys.modules)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "False"


def test_g2_spills_to_g3_and_g3_hits_are_staged_by_the_workers():
    """G2 capped at 4 blocks: registered G2 blocks chain to G3 (a spill op the workers run),
    evicted G2 blocks come back from G3 (a stage op before the onboard) and are registered
    in G2 only once the onboard is reported received."""
    g2 = BlockManager(4, 16, "lru", Tier.G2)
    g3 = BlockManager(32, 16, "lru", Tier.G3, registry=g2.registry)
    L = ConnectorLeader(InstanceLeader.scheduler_side(g2, g3), 16)
    prompt = list(range(64))
    L.create_slot(KvbmRequest("a", prompt))
    L.update_state_after_alloc("a", [0, 1, 2, 3, 4], 0)
    m1 = step(L, 1, {"a": ([], [], 65)})
    assert [o.g1_ids for o in m1.offload] == [[0, 1, 2, 3]] and m1.spill == []
    L.update_connector_output(worker_meta={"offloaded": {1: 1}})
    m2 = step(L, 2, {})
    assert len(m2.spill) == 1 and len(m2.spill[0].g2_ids) == 4
    L.update_connector_output(worker_meta={"spilled": {2: 1}})
    assert L.tier_stats["spilled_to_g3"] == 4
    # a different prompt fills G2 and evicts a's blocks there
    other = list(range(1000, 1064))
    L.create_slot(KvbmRequest("b", other))
    L.update_state_after_alloc("b", [10, 11, 12, 13, 14], 0)
    step(L, 3, {"b": ([], [], 65)})
    L.update_connector_output(worker_meta={"offloaded": {3: 1}})
    assert g2.count_prefix(L.slots["a"].seq.sequence_hashes) == 0
    assert len(step(L, 4, {}).spill) == 1  # b's blocks chain to G3 too; G2 holds them until the copy lands
    L.update_connector_output(worker_meta={"spilled": {4: 1}})
    # a's prompt again: all four blocks come from G3, staged into G2 by the workers
    L.create_slot(KvbmRequest("c", prompt + [5]))
    assert L.get_num_new_matched_tokens("c", 0) == (64, True)
    L.update_state_after_alloc("c", [20, 21, 22, 23, 24], 64)
    m4 = step(L, 5, {})
    [st] = m4.stage
    [ob] = m4.onboard
    assert ob.g2_ids == st.g2_ids and ob.g1_ids == [20, 21, 22, 23]
    assert g2.count_prefix(L.slots["c"].seq.sequence_hashes) == 0  # not matchable before the data lands
    L.update_connector_output(finished_recving={"c"})
    assert g2.count_prefix(L.slots["c"].seq.sequence_hashes) == 4
    assert L.tier_stats["staged_from_g3"] == 4


def test_scheduler_side_leader_refuses_direct_moves():
    """The scheduler-side leader owns G2/G3 state only: a direct onboard or G3 stage
    raises (the bytes move through the connector's workers), it never reports a copy
    that did not happen."""
    g2 = BlockManager(8, 16, "lru", Tier.G2)
    g3 = BlockManager(8, 16, "lru", Tier.G3, registry=g2.registry)
    leader = InstanceLeader.scheduler_side(g2, g3)
    blocks = g2.allocate_blocks(1)
    imm = g2.register_mutable(blocks, [123])
    with pytest.raises(RuntimeError, match="no in-process workers"):
        leader.onboard(imm, [0])
    for b in imm:
        b.release()
    g3b = g3.register_mutable(g3.allocate_blocks(1), [456])
    with pytest.raises(RuntimeError, match="PREPARE"):
        leader.stage_g3_to_g2(g3b)


def test_worker_reports_sent_only_for_requests_that_sent():
    """vLLM frees a finished request at once unless the scheduler delayed it for a send, and
    asserts on a finished_sending report of a request it no longer knows: the worker reports
    only requests it sent blocks for (offloads, pushes)."""
    from kvbm_b200.connector.worker import ConnectorWorker

    w = ConnectorWorker(device=0)
    assert w.get_finished({"a", "b"}) == (set(), set())
    w._send_seen.add("b")  # "b" offloaded; its copies have completed (no events left to wait for)
    assert w.get_finished({"a", "b"}) == ({"b"}, set())
    assert w.get_finished({"b"}) == (set(), set())  # reported once


def test_remote_pull_reports_and_failures():
    """A remote-search pull leaves with the next step's metadata and completes when every worker
    reported it; a worker that could not copy makes the pull fail (the request then prefills)."""
    import threading as th

    g2 = BlockManager(8, 16, "lru", Tier.G2)
    L = ConnectorLeader(InstanceLeader.scheduler_side(g2), 16, num_workers=2)
    res = {}

    def pull(name, **kw):
        try:
            L.queue_remote_pull([{"extra": {}}], [1, 2], [5, 6], timeout=5.0)
            res[name] = "ok"
        except Exception as e:  # noqa: BLE001
            res[name] = type(e).__name__

    t = th.Thread(target=pull, args=("a",))
    t.start()
    while True:
        m = ConnectorMetadata.decode(L.build_connector_meta(SchedulerOutputLite(1)))
        if m.pull:
            break
    [op] = m.pull
    assert (op.src_ids, op.g2_ids) == ([1, 2], [5, 6])
    L.update_connector_output(worker_meta={"pulled": {op.pull_id: 1}})
    assert t.is_alive()  # one of two workers
    L.update_connector_output(worker_meta={"pulled": {op.pull_id: 1}})
    t.join(5)
    assert res["a"] == "ok"
    t = th.Thread(target=pull, args=("b",))
    t.start()
    while not (m := ConnectorMetadata.decode(L.build_connector_meta(SchedulerOutputLite(2)))).pull:
        pass
    L.update_connector_output(worker_meta={"pulled": {m.pull[0].pull_id: 1}, "offloaded": {}})
    L.update_connector_output(worker_meta={"pull_failed": {m.pull[0].pull_id: 1}})
    t.join(5)
    assert res["b"] == "RuntimeError"
