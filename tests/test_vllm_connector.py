"""The vLLM v1 adapter on CPU: the scheduler-role connector, built on vLLM's
real ``KVConnectorBase_V1``, answers the scheduler hooks from a stub
config and stub requests (no engine, no GPU)."""

from types import SimpleNamespace

import pytest
import torch

vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")

from kvbm_b200.connector.protocol import ConnectorMetadata  # noqa: E402


class _ModelConfig:
    dtype = torch.bfloat16
    max_model_len = 4096
    use_mla = False
    hf_config = SimpleNamespace(num_hidden_layers=2)

    def get_num_kv_heads(self, pc):
        return 2

    def get_num_layers(self, pc):
        return 2

    def get_head_size(self):
        return 64


def _vllm_config(extra):
    return SimpleNamespace(
        model_config=_ModelConfig(),
        parallel_config=SimpleNamespace(tensor_parallel_size=1, pipeline_parallel_size=1, rank=0),
        cache_config=SimpleNamespace(block_size=16, cache_dtype="auto"),
        kv_transfer_config=SimpleNamespace(kv_connector="KvbmConnector", kv_role="kv_both",
                                           kv_connector_extra_config=extra))


def _request(rid, tokens):
    return SimpleNamespace(request_id=rid, prompt_token_ids=tokens, cache_salt=None, lora_request=None,
                           kv_transfer_params=None)


def _sched_output(new_reqs, computed, finished=()):
    news = [SimpleNamespace(req_id=r, block_ids=(b,), num_computed_tokens=0) for r, b in new_reqs]
    return SimpleNamespace(scheduled_new_reqs=news, scheduled_cached_reqs=None,
                           num_scheduled_tokens=computed, finished_req_ids=set(finished))


def test_scheduler_role_offloads_then_matches():
    from kvbm_b200.connector import vllm_connector as vc

    Role = vllm_base.KVConnectorRole
    conn = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}}}}), Role.SCHEDULER)
    assert isinstance(conn, vllm_base.KVConnectorBase_V1)
    tokens = list(range(5 * 16 + 3))
    r1 = _request("a", tokens)
    assert conn.get_num_new_matched_tokens(r1, 0) == (0, False)  # cold
    blocks = SimpleNamespace(get_block_ids=lambda: ([10, 11, 12, 13, 14, 15],))
    conn.update_state_after_alloc(r1, blocks, 0)
    meta = conn.build_connector_meta(_sched_output([("a", [10, 11, 12, 13, 14, 15])], {"a": len(tokens)}))
    assert isinstance(meta, vc.KvbmConnectorMetadata)
    m = ConnectorMetadata.decode(meta.metadata)
    assert [op.g1_ids for op in m.offload] == [[10, 11, 12, 13, 14]]  # the five full prompt blocks
    # the worker reports step 1's copies done: only now are the G2 blocks registered
    wm = vc.KvbmConnectorWorkerMetadata({"offloaded": {1: 1}})
    conn.update_connector_output(SimpleNamespace(finished_sending={"a"}, finished_recving=None,
                                                 kv_connector_worker_meta=wm, invalid_block_ids=set()))
    assert conn.request_finished(r1, [10, 11, 12, 13, 14, 15]) == (False, None)

    # the same prompt again: five blocks come from G2 (the last token is always computed)
    r2 = _request("b", tokens)
    assert conn.get_num_new_matched_tokens(r2, 0) == (5 * 16, True)
    conn.update_state_after_alloc(r2, SimpleNamespace(get_block_ids=lambda: ([20, 21, 22, 23, 24, 25],)), 5 * 16)
    m2 = ConnectorMetadata.decode(conn.build_connector_meta(_sched_output([("b", [20, 21, 22, 23, 24, 25])],
                                                                          {"b": 3})).metadata)
    assert len(m2.onboard) == 1 and m2.onboard[0].g1_ids == [20, 21, 22, 23, 24]
    assert conn.build_kv_connector_stats() is None


def test_preempted_request_is_fenced_and_resumes():
    from kvbm_b200.connector import vllm_connector as vc

    Role = vllm_base.KVConnectorRole
    conn = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}}}}), Role.SCHEDULER)
    tokens = list(range(5 * 16 + 3))
    r = _request("p", tokens)
    assert conn.get_num_new_matched_tokens(r, 0) == (0, False)
    conn.update_state_after_alloc(r, SimpleNamespace(get_block_ids=lambda: ([10, 11, 12, 13, 14, 15],)), 0)
    # first chunk: 32 tokens computed -> two full blocks saved
    m1 = ConnectorMetadata.decode(conn.build_connector_meta(
        _sched_output([("p", [10, 11, 12, 13, 14, 15])], {"p": 32})).metadata)
    assert [op.g1_ids for op in m1.offload] == [[10, 11]]
    assert m1.evict == []
    # the scheduler preempts it: the workers are told to fence its offloads
    so = SimpleNamespace(scheduled_new_reqs=[], scheduled_cached_reqs=None, num_scheduled_tokens={},
                         finished_req_ids=set(), preempted_req_ids={"p"})
    m2 = ConnectorMetadata.decode(conn.build_connector_meta(so).metadata)
    assert m2.evict == ["p"] and m2.offload == []
    # resumed with new G1 blocks and recomputed in full: only the blocks not yet in G2 are saved
    cached = SimpleNamespace(req_ids=["p"], new_block_ids=[([30, 31, 32, 33, 34, 35],)], num_computed_tokens=[0],
                             new_token_ids=[[]], all_token_ids={})
    so3 = SimpleNamespace(scheduled_new_reqs=[], scheduled_cached_reqs=cached, num_scheduled_tokens={"p": 83},
                          finished_req_ids=set(), preempted_req_ids=None)
    m3 = ConnectorMetadata.decode(conn.build_connector_meta(so3).metadata)
    assert [op.g1_ids for op in m3.offload] == [[32, 33, 34]]


def test_pd_connector_validates_children_and_routes_handshakes():
    from kvbm_b200.connector import pd
    from kvbm_b200.connector import vllm_connector as vc

    Role = vllm_base.KVConnectorRole
    kvbm = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 8}}}}), Role.SCHEDULER)
    with pytest.raises(ValueError, match="exactly two"):
        pd.validate_children([kvbm])
    with pytest.raises(TypeError, match="first connector"):
        pd.validate_children([object(), kvbm])
    with pytest.raises(TypeError, match="second connector to be NixlConnector"):
        pd.validate_children([kvbm, object()])
    H = pd.PdHandshakeMetadata
    a, b, legacy = object(), object(), object()
    kv, nx = pd.route_handshake({0: H(kvbm_metadata=a, nixl_metadata=b), 1: H(kvbm_metadata=None, nixl_metadata=b),
                                 2: legacy}, H)
    assert kv == {0: a} and nx == {0: b, 1: b, 2: legacy}


def test_disagg_roles_dispatch_over_the_file_plane_and_push(tmp_path):
    """The adapter's disaggregation settings: a decode-role connector sends a prompt to the
    prefill instance over the on-node plane, and a prefill-role connector that receives the
    request (its kv_transfer_params name the decode instance) plans the push of its blocks."""
    from kvbm_b200.connector import vllm_connector as vc
    from kvbm_b200.connector.leader import REMOTE_DECODE_KEY
    from kvbm_b200.engine.cd_plane import FilePeerDirectory, FilePrefillPlane

    Role = vllm_base.KVConnectorRole
    url = f"file://{tmp_path}"
    dec = vc.KvbmConnector(_vllm_config({"disagg": {"role": "decode", "instance_id": 11, "prefill_instance": 22,
                                                    "selection": "always", "directory": url,
                                                    "mailbox_slots": 4}}), Role.SCHEDULER)
    pre = vc.KvbmConnector(_vllm_config({"disagg": {"role": "prefill", "instance_id": 22, "directory": url}}),
                           Role.SCHEDULER)
    # the prefill engine's worker publishes its TP degree when its KV caches are registered
    FilePeerDirectory(str(tmp_path)).publish(22, {"tp": 1, "rank": 0, "instance": 22})
    tokens = list(range(3 * 16 + 5))
    r = _request("d1", tokens)
    assert dec.get_num_new_matched_tokens(r, 0) == (len(tokens), True)  # the whole prompt arrives remotely
    dec.update_state_after_alloc(r, SimpleNamespace(get_block_ids=lambda: ([40, 41, 42, 43],)), len(tokens))
    m = ConnectorMetadata.decode(dec.build_connector_meta(_sched_output([], {})).metadata)
    assert [(op.req_id, op.g1_ids) for op in m.recv] == [("d1", [40, 41, 42, 43])]
    got = FilePrefillPlane(str(tmp_path)).poll(22)
    assert len(got) == 1 and list(got[0]["tokens"]) == tokens
    assert got[0]["decode"]["instance"] == 11 and got[0]["decode"]["dst_ids"] == [40, 41, 42, 43]

    # the prefill engine serves it as a one-token request naming the decode instance
    params = dict(got[0]["params"])
    params[REMOTE_DECODE_KEY] = got[0]["decode"]
    rp = SimpleNamespace(request_id="p1", prompt_token_ids=tokens, cache_salt=None, lora_request=None,
                         kv_transfer_params=params)
    assert pre.get_num_new_matched_tokens(rp, 0) == (0, False)
    pre.update_state_after_alloc(rp, SimpleNamespace(get_block_ids=lambda: ([7, 8, 9, 10],)), 0)
    mp = ConnectorMetadata.decode(pre.build_connector_meta(_sched_output([("p1", [7, 8, 9, 10])],
                                                                         {"p1": len(tokens)})).metadata)
    pushed = [(op.peer, op.src_ids, op.dst_ids) for op in mp.push]
    assert pushed and all(p == 11 for p, _, _ in pushed)
    assert sum((s for _, s, _ in pushed), []) == [7, 8, 9, 10]
    assert sum((d for _, _, d in pushed), []) == [40, 41, 42, 43]
    assert mp.push[-1].final
    # its blocks stay allocated until the workers report the push done
    assert pre.request_finished(rp, [7, 8, 9, 10])[0] is True


def test_disagg_settings_are_validated(tmp_path):
    from kvbm_b200.connector import vllm_connector as vc
    from kvbm_b200.utils.config import KvbmConfig

    def cfg(d):
        return KvbmConfig.for_leader({"disagg": d}, env={}, system_toml=None)

    assert vc.disagg_leader_kwargs(cfg({})) == {}
    with pytest.raises(ValueError, match="instance_id"):
        vc.disagg_leader_kwargs(cfg({"role": "decode"}))
    with pytest.raises(ValueError, match="prefill_instance or hub.url"):
        vc.disagg_leader_kwargs(cfg({"role": "decode", "instance_id": 1, "selection": "always",
                                     "directory": f"file://{tmp_path}"}))
    kw = vc.disagg_leader_kwargs(cfg({"role": "prefill", "instance_id": 2, "directory": f"file://{tmp_path}"}))
    assert kw["instance_id"] == 2 and "cd" not in kw and "plane" not in kw
    with pytest.raises(ValueError, match="directory URL"):
        vc.disagg_leader_kwargs(cfg({"role": "prefill", "instance_id": 2, "directory": "nats://x"}))


def test_scheduler_connector_runs_the_consolidator(monkeypatch):
    """With prefix caching and vLLM KV events configured, the scheduler-role connector starts the
    consolidator: it subscribes to vLLM's event endpoint and republishes deduplicated events on the
    block manager's port + 1000; the enable rules follow the environment and the vLLM config."""
    import socket
    import time

    import msgpack
    import zmq

    from kvbm_b200.connector import consolidator_config as cc
    from kvbm_b200.connector import vllm_connector as vc

    def free_port():
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            return s.getsockname()[1]

    ctx = zmq.Context.instance()
    vpub = ctx.socket(zmq.PUB)
    vport = vpub.bind_to_random_port("tcp://127.0.0.1")
    out_port = free_port()
    monkeypatch.setenv("DYN_KVBM_LEADER_ZMQ_PUB_PORT", str(out_port - 1000))
    cfg = _vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}}}})
    cfg.cache_config.enable_prefix_caching = True
    cfg.kv_events_config = SimpleNamespace(endpoint=f"tcp://*:{vport}")
    cfg.parallel_config.data_parallel_rank = 0
    assert cc.get_consolidator_endpoints(cfg) == (f"tcp://127.0.0.1:{vport}", f"tcp://0.0.0.0:{out_port}",
                                                  f"tcp://127.0.0.1:{out_port}")
    conn = vc.KvbmConnector(cfg, vllm_base.KVConnectorRole.SCHEDULER)
    sub = ctx.socket(zmq.SUB)
    sub.setsockopt(zmq.SUBSCRIBE, b"")
    sub.connect(f"tcp://127.0.0.1:{out_port}")
    try:
        assert conn.consolidator is not None
        stored = {"type": "BlockStored", "block_hashes": [7, 8], "parent_block_hash": None,
                  "token_ids": list(range(32)), "block_size": 16}
        got = []
        deadline = time.monotonic() + 10
        while not got and time.monotonic() < deadline:  # the SUB sockets join asynchronously
            vpub.send_multipart([b"kv", msgpack.packb([time.time(), [stored], None], use_bin_type=True)])
            if sub.poll(200):
                got = msgpack.unpackb(sub.recv_multipart()[-1], raw=False)[1]
        assert [e["type"] for e in got] == ["BlockStored", "BlockStored"]
        assert got[0]["token_ids"] == list(range(16))
    finally:
        conn.shutdown()
        sub.close(0)
        vpub.close(0)
    # opt-out and missing prerequisites
    monkeypatch.setenv("DYN_KVBM_KV_EVENTS_ENABLE_CONSOLIDATOR", "0")
    assert cc.get_consolidator_endpoints(cfg) is None
    monkeypatch.delenv("DYN_KVBM_KV_EVENTS_ENABLE_CONSOLIDATOR")
    cfg.kv_events_config = None
    assert not cc.should_enable_consolidator(cfg)
    pd = _vllm_config({"connectors": [{"kv_connector": "KvbmConnector"}, {"kv_connector": "NixlConnector"}]})
    pd.kv_transfer_config.kv_connector = "PdConnector"
    pd.cache_config.enable_prefix_caching = True
    pd.kv_events_config = SimpleNamespace(endpoint="tcp://*:5557")
    assert cc.should_enable_consolidator(pd)
    assert cc._offset_port("tcp://*:5557", 2) == "tcp://*:5559" and cc._offset_port("inproc://c", 1) == "inproc://c_dp1"
    monkeypatch.setenv("DYN_KVBM_KV_EVENTS_CONSOLIDATOR_MODE", "weird")
    assert cc.get_consolidator_mode() == "dedup"


def test_scheduler_connector_serves_prometheus_metrics():
    """``metrics.enabled``: the scheduler-role connector serves its pools' and cache counters on
    ``metrics.port`` under the reference's metric names."""
    import socket
    import urllib.request

    from kvbm_b200.connector import vllm_connector as vc

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    conn = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}},
                                                     "metrics": {"enabled": True, "port": port},
                                                     "disagg": {"role": "decode", "instance_id": 1,
                                                                "prefill_instance": 2, "selection": "never"}}}),
                            vllm_base.KVConnectorRole.SCHEDULER)
    try:
        conn.get_num_new_matched_tokens(_request("m", list(range(40))), 0)
        body = urllib.request.urlopen(f"http://127.0.0.1:{port}/metrics", timeout=5).read().decode()
        assert 'kvbm_reset_pool_size{tier="g2"} 64.0' in body
        assert "kvbm_allocations_total" in body and "kvbm_host_cache_hit_rate" in body
        assert "kvbm_cd_decisions" in body
    finally:
        conn.shutdown()


def test_scheduler_connector_applies_the_configured_offload_policies():
    """``offload.*.policies`` reach the scheduler's tier engine; an LFU policy gets a frequency
    sketch on the registry, so repeated accesses count."""
    from kvbm_b200.connector import vllm_connector as vc
    from kvbm_b200.engine.offload import PresenceAndLFUFilter, PresenceFilter

    conn = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}},
                                                     "offload": {"g1_to_g2": {"policies": ["presence_lfu"]}}}}),
                            vllm_base.KVConnectorRole.SCHEDULER)
    eng = conn._leader.engine
    assert isinstance(eng.g2_policy, PresenceAndLFUFilter)
    reg = conn._leader.leader.g2.registry
    reg.touch(12345)
    reg.touch(12345)
    assert reg.frequency(12345) >= 2
    plain = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}}}}),
                             vllm_base.KVConnectorRole.SCHEDULER)
    assert isinstance(plain._leader.engine.g2_policy, PresenceFilter)


def test_reference_shaped_vllm_config(capsys):
    """``kvbm.vllm.config.extract_vllm_config_for_kvbm`` returns a ``KvbmVllmConfig`` with the
    reference's parallel / attention sections and prints the table on rank 0."""
    from kvbm.vllm.config import extract_vllm_config_for_kvbm

    from kvbm_b200._core import KvbmVllmConfig

    c = extract_vllm_config_for_kvbm(_vllm_config({}))
    assert isinstance(c, KvbmVllmConfig)
    assert c.parallel["tensor_parallel_size"] == 1 and c.parallel["rank"] == 0
    assert c.attention["block_size"] == 16 and c.attention["head_size"] == 64 and c.attention["num_heads"] == 2
    assert c.attention["cache_dtype_bytes"] == 2 and c.info["block_size"] == 16
    assert "Parallel:" in capsys.readouterr().out
    extract_vllm_config_for_kvbm(_vllm_config({}), log_config=False)
    assert capsys.readouterr().out == ""
    flat = KvbmVllmConfig({"block_size": 16, "rank": 0})
    assert flat.attention == {"block_size": 16} and flat.parallel == {"rank": 0}
