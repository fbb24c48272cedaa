"""Control-plane services on CPU: hub (registry/TTL, indexer, CD queue,
prefill routing with a real prefill handler over the messenger), messenger
RPC/events, config layering, offload pipelines, metrics, strategy matrix."""

import time

import pytest

from kvbm_b200 import _core_native as core
from kvbm_b200.engine.offload import (AllOf, AnyOf, OffloadItem, OffloadPipeline, OffloadState,
                                      PassAll, PresenceAndLFUFilter, PresenceFilter)
from kvbm_b200.hub.client import CompletionEvent, HubClient, HubRegistration, PrefillRouterHandler
from kvbm_b200.hub.kvbmctl import main as kvbmctl
from kvbm_b200.hub.prefill_router import BreakerConfig, BreakerTier, Calibration, CircuitBreaker, Selector
from kvbm_b200.hub.server import HubServer
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.physical.transfer import StorageKind, TransferStrategy, select_strategy, TransferCapabilities
from kvbm_b200.runtime.messenger import EventPoisoned, MessengerPair, RpcError, wait_until
from kvbm_b200.utils.config import KvbmConfig
from kvbm_b200.utils.metrics import KvbmCollector, make_registry


@pytest.fixture
def hub():
    h = HubServer(max_seq_len=4096, ttl=0.3).start()
    yield h
    h.stop()


def test_hub_registry_ttl_and_guard(hub):
    c = HubClient(hub.url)
    assert c.health()["status"] == "ok"
    c.register(11, role="decode", features=["indexer"], address="tcp://x")
    assert [i["instance_id"] for i in c.instances()] == ["11"]
    assert wait_until(lambda: c.instances() == [], 3.0)  # no heartbeat -> evicted after ttl
    with HubRegistration(c, 12, heartbeat_s=0.05, role="prefill") as reg:
        time.sleep(0.6)
        assert [i["instance_id"] for i in c.instances()] == ["12"]  # heartbeats keep it alive
    assert c.instances() == []  # the guard deregistered


def test_hub_indexer_deepest_holder(hub):
    c = HubClient(hub.url)
    for iid in (1, 2):
        c.register(iid, features=["indexer"])
    hs = sequence_hashes(list(range(16 * 6)), 16)
    c.publish_events(1, [("create", hs[:5])])
    c.publish_events(2, [("create", hs[:2])])
    q = c.query(hs)
    assert q["hit"] and q["hash"] == hs[4] and q["holders"] == [1]
    c.publish_events(1, [("remove", hs[2:5])])
    q = c.query(hs)
    assert q["position"] == 1 and sorted(q["holders"]) == [1, 2]
    c.unregister(1)
    assert c.query(hs)["holders"] == [2]


def test_hub_cd_queue_and_dispatch_to_prefill_handler(hub):
    c = HubClient(hub.url)
    c.cd_enqueue({"request_id": "r1", "num_tokens": 100})
    assert c.cd_dequeue()["request_id"] == "r1" and c.cd_dequeue() is None

    seen = []

    def dispatch(req, done: CompletionEvent):
        seen.append(req["request_id"])
        done.complete({"first_token": 42})

    h = PrefillRouterHandler(hub.url, dispatch, calibrate=lambda: {"ttft": [(1000, 0.1), (2000, 0.25),
                                                                           (4000, 0.7)]})
    try:
        assert wait_until(lambda: len(c.targets()) == 1, 3.0)
        out = c.dispatch(4096, 1024, {"request_id": "r2"})
        assert out["forwarded"] and out["result"]["result"] == {"first_token": 42}
        assert seen == ["r2"]
        counters = c.router_counters()
        assert counters["counters"]["dispatched"] == 1
        assert "ttft_coeffs" in counters["calibration"][str(h.instance_id)]
    finally:
        h.close()


def test_kvbmctl_renders(hub, capsys):
    HubClient(hub.url).register(5, role="both", features=["indexer"])
    assert kvbmctl(["--hub", hub.url, "instances"]) == 0
    assert "INSTANCE_ID" in capsys.readouterr().out


def test_kvbmctl_renders_the_vllm_flags(hub, capsys):
    import json
    import shlex

    from kvbm_b200.hub.kvbmctl import render_vllm_cli

    assert kvbmctl(["--hub", hub.url, "config", "vllm", "--features", "disagg", "--role", "decode",
                    "--kvbm", "cache.host.cache_size_gb=4", "--kvbm-config", '{"disagg": {"role": "prefill"}}']) == 0
    line = capsys.readouterr().out.strip()
    toks = shlex.split(line)
    assert toks[:4] == ["--block-size", "16", "--max-model-len", "4096"]
    ktc = json.loads(toks[toks.index("--kv-transfer-config") + 1])
    extra = ktc["kv_connector_extra_config"]
    assert ktc["kv_connector"] == "KvbmConnector" and ktc["kv_load_failure_policy"] == "recompute"
    assert extra["hub"] == {"url": hub.url, "features": ["p2p", "disagg"]}  # dependency pulled in, no router
    assert extra["disagg"]["role"] == "decode"  # the hub-owned role wins over --kvbm-config
    assert extra["cache"]["host"]["cache_size_gb"] == 4
    cfg = {"features": ["indexer", "p2p", "disagg", "prefill_router"], "block_size": 16}
    pre = render_vllm_cli(cfg, "http://h'x", ["disagg"], "prefill")
    assert "prefill_router" in pre and "'\\''" in pre  # router for a prefill role; quote escaped
    with pytest.raises(ValueError):
        render_vllm_cli(cfg, "u", ["disagg"], None)      # disagg needs a role
    with pytest.raises(ValueError):
        render_vllm_cli({"features": ["indexer"]}, "u", ["p2p"])  # not enabled on the hub
    with pytest.raises(ValueError):
        render_vllm_cli(cfg, "u", [], None, ["cache.nope=1"])  # the config loader rejects unknown keys
    assert kvbmctl(["--hub", hub.url, "config", "vllm", "--features", "bogus"]) == 2


def test_selector_and_breaker():
    s = Selector(max_inflight=1)
    s.add_worker(1)
    s.add_worker(2)
    a = s.pick(1000, 0)
    b = s.pick(500, 0)
    assert {a.slot.instance_id, b.slot.instance_id} == {1, 2}
    with pytest.raises(TimeoutError):
        s.pick(10, 0, timeout=0.05)
    a.release()
    c = s.pick(10, 0)
    assert c.slot.instance_id == a.slot.instance_id
    br = CircuitBreaker(BreakerConfig(warm_enter=10, hot_enter=20, warm_exit=5, hot_exit=15))
    assert br.evaluate(12) == BreakerTier.WARM
    assert br.evaluate(25) == BreakerTier.HOT
    assert br.evaluate(16) == BreakerTier.HOT     # hysteresis
    assert br.evaluate(10) == BreakerTier.WARM
    assert br.evaluate(1) == BreakerTier.CALM
    cal = Calibration()
    for x in (100, 200, 400, 800):
        cal.add_ttft(x, 0.01 + 1e-4 * x + 1e-7 * x * x)
    assert abs(cal.predict_ttft(600) - (0.01 + 0.06 + 0.036)) < 1e-6


def test_messenger_rpc_events_and_errors():
    p = MessengerPair()
    try:
        p.b.register_handler("echo", lambda x: x)
        assert p.a.call(p.b.instance_id, "echo", {"k": [1, 2]}) == {"k": [1, 2]}
        with pytest.raises(RpcError):
            p.a.call(p.b.instance_id, "missing")
        ev = p.a.new_event()
        p.b.poison(ev, "pull failed", owner=p.a.instance_id)
        with pytest.raises(EventPoisoned):
            p.a.wait_event(ev, timeout=1)
        with pytest.raises(TimeoutError):
            p.a.wait_event(p.a.new_event(), timeout=0.05)
    finally:
        p.close()


def test_config_layering(tmp_path):
    toml = tmp_path / "k.toml"
    toml.write_text('[cache.host]\ncache_size_gb = 2.0\n[onboard]\nmode = "intra"\n')
    env = {"DYN_KVBM_CPU_CACHE_GB": "1", "KVBM_CONFIG_PATH": str(toml), "KVBM_CACHE_DISK_NUM_BLOCKS": "7"}
    c = KvbmConfig.load({"default": {"block_size": 32}, "worker": {"cache": {"host": {"num_blocks": 9}}}},
                        role="worker", env=env, system_toml=None)
    assert c.cache.host.cache_size_gb == 2.0       # TOML beats DYN_KVBM_*
    assert c.cache.disk.num_blocks == 7            # KVBM_* env
    assert c.cache.host.num_blocks == 9            # JSON worker profile
    assert c.block_size == 32 and c.onboard.mode == "intra"
    with pytest.raises(ValueError):
        KvbmConfig.load({"block_layout": "weird"}, env={}, system_toml=None)
    with pytest.raises(ValueError):
        KvbmConfig.load({"nonsense": 1}, env={}, system_toml=None)
    c = KvbmConfig.load({"leader": {"remote_search": {"enabled": True, "min_remote_tokens": 64}}}, role="leader",
                        env={"KVBM_MESSENGER_BIND": "tcp://0.0.0.0:5555"}, system_toml=None)
    assert c.remote_search.enabled and c.remote_search.min_remote_tokens == 64
    assert c.messenger.bind == "tcp://0.0.0.0:5555" and c.messenger.discovery == "hub"


def test_offload_pipeline_policies_batching_cancel():
    dst = BlockManager(32, 16, "lru", Tier.G2, registry=core.Registry(frequency=core.TinyLfu(64)))
    calls = []

    def executor(items):
        calls.append(len(items))
        blocks = dst.allocate_blocks(len(items))
        return dst.register_mutable(blocks, [i.seq_hash for i in items])

    hs = sequence_hashes(list(range(16 * 10)), 16)
    p = OffloadPipeline("g1_to_g2", dst, executor, PresenceFilter(dst))
    p.cfg.max_batch = 4
    h = p.enqueue([OffloadItem(x, i) for i, x in enumerate(hs[:6])])
    assert h.wait(5) == OffloadState.DONE and calls == [4, 2]
    h2 = p.enqueue([OffloadItem(x, i) for i, x in enumerate(hs[:8])])
    assert h2.wait(5) == OffloadState.DONE and len(h2.skipped) == 6  # presence filter
    gate = {"open": False}
    h3 = p.enqueue([OffloadItem(hs[9], 9)], precondition=lambda: gate["open"])
    time.sleep(0.05)
    assert h3.cancel() and h3.wait(5) == OffloadState.CANCELLED
    assert not h2.cancel()  # already final
    lfu = PresenceAndLFUFilter(dst, min_frequency=3)
    assert not lfu.keep(OffloadItem(hs[9], 0))
    assert AnyOf(PassAll(), lfu).keep(OffloadItem(hs[9], 0)) and not AllOf(PassAll(), lfu).keep(OffloadItem(hs[9], 0))
    p.close()


def test_metrics_collector_names():
    mgr = BlockManager(8, 16, "lru", Tier.G2)
    blocks = mgr.allocate_blocks(2)
    mgr.register_mutable(blocks, sequence_hashes(list(range(32)), 16))
    col = KvbmCollector()
    col.add_pool("g2", mgr)
    col.transfer.observe(0.002, 1 << 20)
    from prometheus_client import generate_latest

    text = generate_latest(make_registry(col)).decode()
    for name in ("kvbm_allocations_total", "kvbm_registrations_total", "kvbm_inactive_pool_size",
                 "kvbm_transfer_duration_seconds_bucket", "kvbm_host_cache_hit_rate", "kvbm_cd_decisions_total"):
        assert name in text, name


def test_strategy_matrix():
    K, S = StorageKind, TransferStrategy
    assert select_strategy(K.PINNED, K.DEVICE).first == S.KERNEL_H2D
    assert select_strategy(K.DEVICE, K.PINNED, TransferCapabilities(prefer_copy_engine=True)).first == S.CUDA_ASYNC_D2H
    p = select_strategy(K.DEVICE, K.DISK)
    assert p.is_two_hop and p.bounce == K.PINNED and p.second == S.DISK_WRITE
    assert not select_strategy(K.DEVICE, K.DISK, TransferCapabilities(allow_gds=True)).is_two_hop
    assert select_strategy(K.DEVICE, K.PEER).first == S.KERNEL_P2P
    assert select_strategy(K.DISK, K.DISK).first == S.INVALID


def test_disk_pool_roundtrip(tmp_path):
    import numpy as np

    d = core.DiskPool(str(tmp_path / "g3.bin"), 8, 4096, direct=False, persistent=True)
    a = np.random.randint(0, 255, 4096 * 3, dtype=np.uint8)
    b = np.zeros_like(a)
    d.write([1, 4, 7], [a.ctypes.data + i * 4096 for i in range(3)])
    d.read([1, 4, 7], [b.ctypes.data + i * 4096 for i in range(3)])
    assert (a == b).all() and d.bytes_written() == 3 * 4096
    with pytest.raises(IndexError):
        d.read([8], [b.ctypes.data])


def test_tier_journal_restores_g3_registrations(tmp_path):
    from kvbm_b200.engine.tier_journal import TierJournal, restore

    path = str(tmp_path / "g3.journal")
    hs = sequence_hashes(list(range(16 * 6)), 16)
    j = TierJournal(path)
    j.invalidate([0, 1, 2])
    j.commit([0, 1, 2], hs[:3])
    j.invalidate([1])            # block 1 is being overwritten ...
    j.commit([4], hs[3:4])
    j.invalidate([5])            # ... and block 5's write never completed (crash)
    j.close()
    with open(path, "ab") as f:
        f.write(b"\x85\xa2op")   # torn tail
    live = TierJournal.replay(path)
    assert live == {0: hs[0], 2: hs[2], 4: hs[3]}
    g3 = BlockManager(8, 16, "lru", Tier.G3)
    assert restore(g3, live) == 3
    got = g3.match_blocks(hs[:1])
    assert [b.block_id for b in got] == [0]
    for b in got:
        b.release()
    assert g3.allocate_blocks(5) is not None  # the 5 unjournaled ids were freed
    j2 = TierJournal(path)
    j2.compact()
    assert TierJournal.replay(path) == live
    j2.close()
    with pytest.raises(RuntimeError):
        restore(g3, live)  # not a fresh pool


def test_hub_control_port_and_cli_settings():
    import requests

    h = HubServer(max_seq_len=1024, control_port=0, layout="universal", advertise_host="10.0.0.7",
                  g2_memory_gb=4.0).start()
    try:
        ctl = f"http://127.0.0.1:{h.control_port}"
        assert h.control_port and h.control_port != h.port
        assert requests.get(ctl + "/health", timeout=5).json()["status"] == "ok"
        cfg = requests.get(h.url + "/v1/config", timeout=5).json()
        assert cfg["layout"] == "universal" and cfg["advertise_host"] == "10.0.0.7" and cfg["g2_memory_gb"] == 4.0
        assert cfg["messenger"].startswith("tcp://")
        # registration and indexer routes are not on the control port
        assert requests.post(ctl + "/v1/indexer/query", json={"hashes": []}, timeout=5).status_code == 404
    finally:
        h.stop()


def test_runtime_registers_with_hub_and_static_peers():
    import json as _json

    import kvbm._core as kc

    h = HubServer(max_seq_len=1024).start()
    try:
        cfg = {"hub": {"url": h.url, "heartbeat_secs": 0.2},
               "messenger": {"peers": {"77": "tcp://127.0.0.1:5999"}}}
        rt = kc.KvbmRuntime.build_leader(_json.dumps(cfg))
        try:
            assert rt.messenger._peers[77] == "tcp://127.0.0.1:5999"
            rt.register_with_hub(features=["indexer", "p2p"])
            got = {int(i["instance_id"]): i for i in HubClient(h.url).instances()}
            assert rt.messenger.instance_id in got and got[rt.messenger.instance_id]["address"] == rt.messenger.address
        finally:
            rt.shutdown()
        assert rt.messenger.instance_id not in {int(i["instance_id"]) for i in HubClient(h.url).instances()}
    finally:
        h.stop()


def test_hub_serves_its_web_ui(hub):
    import requests

    page = requests.get(hub.url + "/", timeout=5)
    assert page.status_code == 200 and "text/html" in page.headers["content-type"]
    assert '<script src="/app.js">' in page.text
    js = requests.get(hub.url + "/app.js", timeout=5)
    assert js.status_code == 200 and "/v1/instances" in js.text and "javascript" in js.headers["content-type"]
    # every element id the script fills exists on the page
    import re

    for el in set(re.findall(r'fill(?:Dl|Table)\("([a-z_]+)"', js.text)):
        assert f'id="{el}"' in page.text, el
    assert requests.get(hub.url + "/style.css", timeout=5).headers["content-type"].startswith("text/css")


def test_kvbmctl_indexer_and_disagg_groups(hub, capsys, monkeypatch):
    """kvbmctl's indexer group (config, get-instances, by-pos, query) and disagg instances, with the
    hub URL taken from KVBMCTL_HUB."""
    import json

    from kvbm_b200.hub.client import HubClient
    from kvbm_b200.hub.kvbmctl import main as kvbmctl
    from kvbm_b200.logical.sequence import sequence_hashes

    c = HubClient(hub.url)
    c.register(91, features=["indexer"], address="tcp://127.0.0.1:1")
    c.register(92, role="prefill", features=["prefill_router"], address="tcp://127.0.0.1:2")
    hs = sequence_hashes(list(range(3 * 16)), 16)
    c.publish_events(91, [("create", hs)])
    monkeypatch.setenv("KVBMCTL_HUB", hub.url)

    def run(*args):
        assert kvbmctl(["--json", *args]) == 0
        return json.loads(capsys.readouterr().out)

    assert run("indexer", "config")["entries"] == 3
    assert "91" in run("indexer", "get-instances")["instances"]
    pos = run("indexer", "by-pos", "2")
    assert pos["position"] == 2 and len(pos["blocks"]) == 1 and pos["blocks"][0]["holders"] == ["91"]
    assert int(pos["blocks"][0]["lineage"]) == hs[2] & ((1 << 64) - 1)
    q = run("indexer", "query", hex(hs[2]))
    assert q["hit"] and q["holders"] == [91] and q["position"] == 2
    assert run("indexer", "by-pos", "7")["blocks"] == []
    assert "92" in run("disagg", "instances")["prefill"]
