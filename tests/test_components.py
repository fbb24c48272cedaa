"""CPU tests: consolidator service over ZeroMQ, G4 object store, conditional
disaggregation policy, KV dimension probing, the ``kvbm._core`` surface."""

import time

import msgpack
import numpy as np
import pytest
import zmq

from kvbm_b200.connector.dim_probe import KvDim, derive_block_layout, infer_from_shape, probe_kv_dim_layout
from kvbm_b200.consolidator.service import Consolidator, source_id
from kvbm_b200.engine.cd import ConditionalDisagg, Decision, InflightBudget, RemotePrefillParams, SelectionPolicy
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.object.store import FsObjectStore
from kvbm_b200.physical.layout import KvBlockLayout
from kvbm_b200.utils.metrics import CdMetrics


def _vllm_batch(events):
    return msgpack.packb([time.time(), events, None], use_bin_type=True)


def test_consolidator_dedups_engine_and_kvbm_sources():
    c = Consolidator("tcp://127.0.0.1:0", block_size=4)
    sub = zmq.Context.instance().socket(zmq.SUB)
    sub.setsockopt(zmq.SUBSCRIBE, b"")
    sub.connect(c.endpoint)
    time.sleep(0.2)
    stored = {"type": "BlockStored", "block_hashes": [111, 222], "parent_block_hash": None,
              "token_ids": list(range(8)), "block_size": 4}
    c.ingest_engine_batch(_vllm_batch([stored]), "vllm")
    c.ingest_engine_batch(_vllm_batch([stored]), "trtllm")  # second source: no new STORE
    out = c.flush()
    assert [e["type"] for e in out] == ["BlockStored", "BlockStored"]
    assert out[1]["parent_block_hash"] == out[0]["block_hashes"][0]
    # the wire message reached the subscriber
    assert sub.poll(2000)
    topic, payload = sub.recv_multipart()
    ts, events, dp = msgpack.unpackb(payload, raw=False)
    assert len(events) == 2 and events[0]["block_size"] == 4
    c.ingest_engine_batch(_vllm_batch([{"type": "BlockRemoved", "block_hashes": [111, 222]}]), "vllm")
    assert c.flush() == []  # trtllm still holds them
    c.ingest_engine_batch(_vllm_batch([["BlockRemoved", [111, 222], None]]), "trtllm")
    assert [e["type"] for e in c.flush()] == ["BlockRemoved", "BlockRemoved"]
    c.ingest_engine_batch(b"\xc1not-msgpack", "vllm")
    assert c.stats["bad_batches"] == 1
    c.ingest_engine_batch(_vllm_batch([{"type": "AllBlocksCleared"}]), "vllm")
    assert c.flush()[-1]["type"] == "AllBlocksCleared"
    with pytest.raises(ValueError):
        source_id("gpu2")
    sub.close(0)
    c.close()


def test_object_store_put_get_lock(tmp_path):
    s = FsObjectStore(str(tmp_path))
    h = sequence_hashes(list(range(16)), 16)[0]
    k = s.key(h, rank=1)
    assert not s.has(k) and s.get(k) is None
    assert s.try_lock(k) and not s.try_lock(k)
    buf = np.arange(4096, dtype=np.uint8)
    [f.result() for f in s.put_blocks([k], [buf.ctypes.data], 4096)]
    assert s.has(k) and s.try_lock(k)  # put released the lock
    out = np.zeros_like(buf)
    assert s.get_blocks([k, k + "x"], [out.ctypes.data, out.ctypes.data], 4096) == [True, False]
    assert (out == buf).all()
    s.close()


def test_conditional_disagg_policy_budget_and_breaker():
    assert SelectionPolicy("threshold", 100).decide(1000, computed=850, connector=100) == Decision.LOCAL
    assert SelectionPolicy("threshold", 100).decide(1000, computed=500) == Decision.REMOTE
    m = CdMetrics()
    cd = ConditionalDisagg(SelectionPolicy("always"), InflightBudget(2), metrics=m)
    assert cd.decide(100) == Decision.REMOTE and cd.decide(100) == Decision.REMOTE
    assert cd.decide(100) == Decision.LOCAL  # budget exhausted
    cd.finish_remote()
    cd.breaker_tier = 2
    assert cd.decide(100) == Decision.LOCAL  # hot breaker forces local
    cd.breaker_tier = 1
    assert cd.decide(100) == Decision.LOCAL  # warm halves the budget (1 in flight already)
    assert m.decisions["remote"] == 2
    p = RemotePrefillParams(initiator_instance_id="7", num_provided_tokens=64)
    assert RemotePrefillParams.from_dict(p.to_dict()) == p


def test_dim_probe_labels_common_backends():
    flash = probe_kv_dim_layout(lambda nb, bs, h, d: (2, nb, bs, h, d))
    assert flash == [KvDim.OUTER, KvDim.BLOCK, KvDim.PAGE, KvDim.HEAD, KvDim.HEAD_SIZE]
    dl = derive_block_layout(flash)
    assert not dl.block_first and dl.inner == KvBlockLayout.OPERATIONAL_NHD
    finfer = probe_kv_dim_layout(lambda nb, bs, h, d: (nb, 2, h, bs, d))
    dl = derive_block_layout(finfer)
    assert dl.block_first and dl.inner == KvBlockLayout.OPERATIONAL_HND
    assert infer_from_shape((2, 100, 16, 8, 128), 100, 16, 8, 128)[0] == KvDim.OUTER
    assert infer_from_shape((100, 32, 2, 16, 8, 128), 100, 16, 8, 128, num_layers=32)[:3] == [
        KvDim.BLOCK, KvDim.LAYER, KvDim.OUTER]
    # two layers, two KV heads: the sizes alone are ambiguous; the cross-layer convention decides
    assert infer_from_shape((40, 2, 2, 16, 2, 128), 40, 16, 2, 128, num_layers=2) == [
        KvDim.BLOCK, KvDim.LAYER, KvDim.OUTER, KvDim.PAGE, KvDim.HEAD, KvDim.HEAD_SIZE]


def test_core_surface_leader_from_layout():
    import kvbm._core as kc
    from kvbm_b200.connector.protocol import ConnectorMetadata

    rt = kc.KvbmRuntime.build_leader('{"cache": {"host": {"num_blocks": 32}}}')
    try:
        iid, addr = rt.peer_info()
        assert len(rt.instance_id()) == 16 and addr.startswith("tcp://")
        leader = kc.ConnectorLeader(rt, 16)
        with pytest.raises(RuntimeError):
            leader.get_num_new_matched_tokens("x", 0)
        leader.initialize_workers(layout={"g2_blocks": 32, "g3_blocks": 0})
        leader.create_slot(kc.KvbmRequest("r", list(range(48))))
        assert leader.get_num_new_matched_tokens("r", 0) == (0, False)
        leader.update_state_after_alloc("r", [4, 5, 6], 0)
        so = kc.SchedulerOutput(1)
        so.add_new_request("r", list(range(48)), [], 0)
        so.add_num_scheduled_tokens({"r": 48})
        meta = ConnectorMetadata.decode(leader.build_connector_metadata(so))
        assert meta.offload[0].g1_ids == [4, 5, 6]
        assert kc.hub.CompletionEvent is not None
        # the leader's control plane answers on the runtime's messenger
        from kvbm_b200.engine.control import LeaderControlClient
        from kvbm_b200.runtime.messenger import Messenger

        m = Messenger()
        try:
            ctl = LeaderControlClient(m, addr)
            assert ctl.list_modules() == ["core", "dev", "metrics"]
            d = ctl.describe()
            assert d["block_size"] == 16 and d["tier_capacity"] == [{"tier": "g2", "total_blocks": 32}]
            assert d["config"]["cache"]["host"]["num_blocks"] == 32
            assert ctl.metrics()["pools"][0]["total_blocks"] == 32
        finally:
            m.close()
    finally:
        rt.shutdown()


def test_host_memory_service_over_grpc(tmp_path):
    from kvbm_b200.service.client import KvbmServiceClient, ServiceError
    from kvbm_b200.service.server import serve

    sock = str(tmp_path / "kvbm.sock")
    server, svc = serve(sock, directory=str(tmp_path))
    try:
        a = KvbmServiceClient(sock)
        b = KvbmServiceClient(sock)
        assert a.health()["status"] == "ok"
        pa = a.create_pool("g2", 8, 4096)
        ids = a.allocate("g2", 3)
        assert ids == [0, 1, 2] and a.allocate("g2", 6) is None
        pa.block(ids[1])[:4] = b"kvbm"
        h = sequence_hashes(list(range(16)), 16)[0]
        a.register("g2", [h], [ids[1]])
        pb = b.create_pool("g2", 8, 4096)  # a second process maps the same pool
        [slot] = b.lookup("g2", [h])
        assert slot == ids[1] and bytes(pb.block(slot)[:4]) == b"kvbm"
        assert b.free("g2", ids) == 8 and b.lookup("g2", [h]) == [-1]
        with pytest.raises(ServiceError):
            b.allocate("nope", 1)
        assert a.stats()["g2"]["free"] == 8
        pa.close()
        pb.close()
    finally:
        server.stop(0)
        svc.close()


def test_events_manager_batches_to_sinks():
    from kvbm_b200.logical.events import EventsManager
    from kvbm_b200.logical.manager import BlockManager, Tier

    em = EventsManager(instance_id=9, policy="all", window_ms=5)
    got = []
    em.add_sink(lambda iid, batches: got.append((iid, batches)))
    mgr = BlockManager(8, 16, "lru", Tier.G2, registry=em.registry())
    blocks = mgr.allocate_blocks(3)
    imm = mgr.register_mutable(blocks, sequence_hashes(list(range(48)), 16))
    em.start()
    time.sleep(0.1)
    em.stop()
    assert got and got[0][0] == 9 and got[0][1][0][0] == "create" and len(got[0][1][0][1]) == 3
    del imm


def test_core_binding_method_names():
    """The ``kvbm._core`` classes answer the reference binding's method names: runtime handler
    waits between two runtimes, scheduler-output accessors and serialisation, slot token access
    on the leader, and the worker hooks."""
    import msgpack

    import kvbm._core as kc

    worker_rt = kc.KvbmRuntime.build_worker('{"cache": {"host": {"num_blocks": 8}}}')
    leader_rt = kc.KvbmRuntime.build_leader('{"cache": {"host": {"num_blocks": 8}}}')
    try:
        wid, waddr = worker_rt.peer_info()
        leader_rt.register_peer(wid, waddr)
        w = kc.ConnectorWorker(worker_rt, block_size=16, num_kv_heads=2, head_size=64)
        leader_rt.wait_for_handler(wid, "kvbm.connector.worker.get_layout_config", timeout_s=5)
        with pytest.raises(TimeoutError):
            leader_rt.wait_for_handler(wid, "no.such.handler", timeout_s=0.3)
        assert not w.is_initialized()
        for name in ("bind_connector_metadata", "clear_connector_metadata", "start_load_kv", "wait_for_layer_load",
                     "save_kv_layer", "wait_for_save", "get_finished", "get_failed_onboarding", "handle_preemptions",
                     "handshake_metadata", "shutdown", "register_kv_caches", "register_cross_layers_kv_cache"):
            assert callable(getattr(kc.ConnectorWorker, name)), name

        so = kc.SchedulerOutput(3)
        so.add_new_request("r", list(range(32)), [1, 2], 0)
        so.set_num_scheduled_tokens({"r": 32})
        so.set_preempted_req_ids({"p"})
        assert so.get_total_num_scheduled_tokens() == 32
        d = msgpack.unpackb(so.serialize(), raw=False)
        assert d["iteration"] == 3 and d["scheduled"]["r"][1] == [1, 2] and d["preempted"] == ["p"]
        assert so.lite().preempted_req_ids == ["p"]

        leader = kc.ConnectorLeader(leader_rt, 16)
        leader.initialize_workers(layout={"g2_blocks": 8, "g3_blocks": 0})
        leader.create_slot(kc.KvbmRequest("r", list(range(20))))
        leader.extend_slot_tokens("r", [7, 8, 9])
        assert leader.get_slot_total_tokens("r") == 23 and leader.block_size == 16
        assert leader.build_connector_meta == leader.build_connector_metadata
    finally:
        worker_rt.shutdown()
        leader_rt.shutdown()


def test_core_leader_takes_the_disaggregation_settings(tmp_path):
    """``kvbm._core.ConnectorLeader`` built from a decode-role configuration dispatches remote
    prefills over the configured plane, like the vLLM adapter."""
    import json

    import kvbm._core as kc
    from kvbm_b200.engine.cd_plane import FilePeerDirectory, FilePrefillPlane

    cfg = {"cache": {"host": {"num_blocks": 16}},
           "disagg": {"role": "decode", "instance_id": 5, "prefill_instance": 6, "selection": "always",
                      "directory": f"file://{tmp_path}", "mailbox_slots": 2}}
    rt = kc.KvbmRuntime.build_leader(json.dumps(cfg))
    try:
        FilePeerDirectory(str(tmp_path)).publish(6, {"tp": 1, "rank": 0, "instance": 6})
        leader = kc.ConnectorLeader(rt, 16)
        leader.initialize_workers(layout={"g2_blocks": 16, "g3_blocks": 0})
        leader.create_slot(kc.KvbmRequest("d", list(range(40))))
        assert leader.get_num_new_matched_tokens("d", 0) == (40, True)
        leader.update_state_after_alloc("d", [1, 2, 3], 40)
        [got] = FilePrefillPlane(str(tmp_path)).poll(6)
        assert got["request_id"] == "d" and got["decode"]["instance"] == 5
    finally:
        rt.shutdown()
