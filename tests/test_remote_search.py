"""Remote search on CPU: instance B finds instance A's prefix through the hub
indexer, pulls it from A's shared-memory G2 pool (or over the messenger),
and the connector stalls the request until the blocks are local."""


import pytest

from kvbm_b200.connector.leader import ConnectorLeader, KvbmRequest
from kvbm_b200.engine.leader import InstanceLeader, ParallelWorkers
from kvbm_b200.engine.remote_search import RemoteHolder, RemoteSearch, RemoteSearchConfig
from kvbm_b200.hub.client import HubClient
from kvbm_b200.hub.server import HubServer
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
from kvbm_b200.physical.verify import FillPattern, checksum_blocks, fill_blocks
from kvbm_b200.runtime.messenger import Messenger

BS = 16


class _Instance:
    def __init__(self, iid, hub, block_layout, shared=True):
        self.iid = iid
        self.g2 = BlockManager(32, BS, "lru", Tier.G2)
        self.leader = InstanceLeader(self.g2, ParallelWorkers([]), instance_id=iid)
        cfg = LayoutConfig.for_model(32, 2, 2, 64, BS)
        self.layout = KvLayout.allocate(cfg, "fully_contiguous", block_layout, location="shared")
        self.msg = Messenger(iid)
        # shared=False: the pool is exported without its file (as across nodes)
        self.holder = RemoteHolder(self.leader, [self.layout], self.msg, shareable=shared)
        hub.register(iid, features=["indexer", "p2p"], address=self.msg.address)

    def close(self):
        self.msg.close()
        self.layout.backing.close()


@pytest.fixture
def hub():
    h = HubServer(max_seq_len=4096).start()
    yield h
    h.stop()


@pytest.mark.parametrize("shared", [True, False])
def test_cold_instance_pulls_prefix_from_holder(hub, shared):
    c = HubClient(hub.url)
    a = _Instance(101, c, KvBlockLayout.OPERATIONAL_NHD, shared=shared)
    b = _Instance(202, c, KvBlockLayout.OPERATIONAL_HND)
    try:
        tokens = list(range(1000, 1000 + 6 * BS + 5))
        hashes = sequence_hashes(tokens, BS)
        # A computed the prompt: 6 full blocks in its G2, announced to the indexer
        blocks = a.g2.allocate_blocks(6)
        fill_blocks(a.layout, [x.block_id for x in blocks], FillPattern.RANDOM, seed=9)
        imm = a.g2.register_mutable(blocks, hashes[:6])
        want = checksum_blocks(a.layout, [x.block_id for x in imm])
        for x in imm:
            x.release()
        c.publish_events(a.iid, [("create", hashes[:6])])

        rs = RemoteSearch(b.leader, [b.layout], b.msg, c, BS, RemoteSearchConfig(enabled=True))
        conn = ConnectorLeader(b.leader, BS, remote_search=rs)
        conn.create_slot(KvbmRequest("r1", tokens))
        assert conn.get_num_new_matched_tokens("r1", 0) == (None, False)  # stalled on the pull
        conn.slots["r1"].remote_future.result(timeout=10)
        n, async_load = conn.get_num_new_matched_tokens("r1", 0)
        assert (n, async_load) == (6 * BS, True)
        got = checksum_blocks(b.layout, [x.block_id for x in conn.slots["r1"].matched])
        assert got == want  # same bytes, NHD on A, HND on B
        assert rs.stats["pulled_blocks"] == 6 and (rs.stats["rpc_reads"] == 0) == shared
        assert a.holder.open_sessions() == 0 and len(a.holder.sessions) == 0
        # A's blocks were released by the session close: all 32 allocatable again
        assert a.g2.allocate_blocks(32) is not None

        # a second request on B is a plain local hit (no new search)
        conn.create_slot(KvbmRequest("r2", tokens))
        assert conn.get_num_new_matched_tokens("r2", 0) == (6 * BS, True)
        assert rs.stats["searches"] == 1
        rs.close()
    finally:
        a.close()
        b.close()


def test_warm_and_unknown_prefixes_skip_or_miss(hub):
    c = HubClient(hub.url)
    a = _Instance(303, c, KvBlockLayout.OPERATIONAL_NHD)
    try:
        rs = RemoteSearch(a.leader, [a.layout], a.msg, c, BS, RemoteSearchConfig(enabled=True,
                                                                                   min_remote_tokens=3 * BS))
        hashes = sequence_hashes(list(range(5 * BS)), BS)
        # only this instance holds the prefix: the self filter leaves no holder
        c.publish_events(a.iid, [("create", hashes[:2])])
        assert rs.search(hashes) is None
        assert rs.search(sequence_hashes(list(range(7, 7 + 5 * BS)), BS)) is None
        # decimated query over a long prompt still finds the deepest probed block
        long_h = sequence_hashes(list(range(200 * BS)), BS)
        rs.config.max_query_hashes = 16
        assert len(rs._query_set(long_h)) <= 17 and rs._query_set(long_h)[-1] == long_h[-1]
        rs.close()
    finally:
        a.close()


def test_kvbmctl_p2p_pin_pull_unpin_and_xfer(hub, capsys):
    import json

    from kvbm_b200.hub.kvbmctl import main as kvbmctl

    c = HubClient(hub.url)
    a = _Instance(401, c, KvBlockLayout.OPERATIONAL_NHD)
    b = _Instance(402, c, KvBlockLayout.OPERATIONAL_HND)
    try:
        hashes = sequence_hashes(list(range(500, 500 + 4 * BS)), BS)
        blocks = a.g2.allocate_blocks(4)
        fill_blocks(a.layout, [x.block_id for x in blocks], FillPattern.RANDOM, seed=3)
        imm = a.g2.register_mutable(blocks, hashes)
        want = checksum_blocks(a.layout, [x.block_id for x in imm])
        for x in imm:
            x.release()
        rs = RemoteSearch(b.leader, [b.layout], b.msg, c, BS, RemoteSearchConfig(enabled=True))
        hs = ",".join(hex(h) for h in hashes[:2])
        assert kvbmctl(["--hub", hub.url, "--json", "p2p", "pin", "--instance-id", "401", "--hashes", hs]) == 0
        pin = json.loads(capsys.readouterr().out)
        assert pin["sid"] is not None and len(pin["block_ids"]) == 2 and a.holder.open_sessions() == 1
        assert kvbmctl(["--hub", hub.url, "--json", "p2p", "pull", "--from", "401", "--to", "402",
                        "--session", json.dumps(pin)]) == 0
        assert json.loads(capsys.readouterr().out) == {"pulled": 2}
        assert a.holder.open_sessions() == 1  # pull leaves the session pinned
        assert kvbmctl(["--hub", hub.url, "--json", "p2p", "unpin", "--instance-id", "401",
                        "--session", pin["sid"]]) == 0
        capsys.readouterr()
        assert a.holder.open_sessions() == 0
        assert kvbmctl(["--hub", hub.url, "--json", "p2p", "xfer", "--from", "401", "--to", "402",
                        "--hashes", ",".join(hex(h) for h in hashes)]) == 0
        assert json.loads(capsys.readouterr().out) == {"pulled": 4}
        got = b.g2.match_blocks(hashes)
        assert checksum_blocks(b.layout, [x.block_id for x in got]) == want
        assert a.holder.open_sessions() == 0
        rs.close()
    finally:
        a.close()
        b.close()


def test_leader_control_plane_modules(hub):
    from kvbm_b200.engine.control import ControlError, LeaderControl, LeaderControlClient, plan_reset

    assert plan_reset(None, {"g2"}) == (["g2"], ["g3"])
    assert plan_reset(["g2", "g2"], {"g2", "g3"}) == (["g2"], [])
    with pytest.raises(ControlError) as e:
        plan_reset(["g2", "g3"], {"g2"})
    assert e.value.kind == "tier_not_configured"
    c = HubClient(hub.url)
    a = _Instance(501, c, KvBlockLayout.OPERATIONAL_NHD)
    b = _Instance(502, c, KvBlockLayout.OPERATIONAL_NHD)
    try:
        rs = RemoteSearch(b.leader, [b.layout], b.msg, c, BS, RemoteSearchConfig(enabled=True))
        LeaderControl(a.leader, a.msg, BS, [{"g2": a.layout}], holder=a.holder, search=None, role="decode",
                      parallelism={"tp": 1})
        ctl_b = LeaderControl(b.leader, b.msg, BS, [{"g2": b.layout}], holder=b.holder, search=rs)
        cli_a, cli_b = LeaderControlClient(b.msg, a.msg.address), LeaderControlClient(a.msg, b.msg.address)
        assert cli_a.list_modules() == ["core", "dev", "metrics"]
        assert cli_b.list_modules() == ["core", "dev", "metrics", "transfer"] == ctl_b.modules
        d = cli_a.describe()
        assert d["instance_id"] == "501" and d["block_size"] == BS and d["role"] == "decode"
        assert d["tier_capacity"] == [{"tier": "g2", "total_blocks": 32}]
        assert d["workers"][0]["layouts"][0]["config"]["num_blocks"] == 32
        hashes = sequence_hashes(list(range(700, 700 + 3 * BS)), BS)
        imm = a.g2.register_mutable(a.g2.allocate_blocks(3), hashes)
        for x in imm:
            x.release()
        c.publish_events(a.iid, [("create", hashes)])
        m = cli_a.metrics()
        assert m["pools"][0]["inactive_blocks"] == 3 and m["sessions_inflight"] == 0
        assert cli_b.search_prefix(hashes) == {"local_g2_blocks": 0, "remote": {"holder": 501, "blocks": 3}}
        # transfer module under its control-plane names: pin on A, pull into B, unpin
        with pytest.raises(ControlError) as e:
            cli_a.open_session(hashes)  # A offers no transfer module
        assert e.value.kind == "module_not_offered"
        opened = LeaderControlClient(a.msg, b.msg.address)  # B's own holder has nothing to pin
        assert opened.open_session(hashes)["sid"] is None
        assert cli_b.pull_from_session(501, {}, hashes) == {"pulled": 3}  # no session: pin + pull + unpin
        assert b.g2.count_prefix(hashes) == 3
        import json

        from kvbm_b200.hub.kvbmctl import main as kvbmctl

        assert kvbmctl(["--hub", hub.url, "--json", "control", "--instance-id", "501", "modules"]) == 0
        assert kvbmctl(["--hub", hub.url, "control", "--instance-id", "501", "reset", "--tiers", "g3"]) == 2
        assert kvbmctl(["--hub", hub.url, "--json", "control", "--instance-id", "501", "reset"]) == 0
        assert a.g2.inactive_len() == 0
        imm = a.g2.register_mutable(a.g2.allocate_blocks(1), hashes[:1])
        imm[0].release()
        r = cli_a.reset()
        assert r == {"reset": ["g2"], "failed": [], "skipped_unconfigured": ["g3"]}
        assert a.g2.inactive_len() == 0
        with pytest.raises(ControlError) as e:
            cli_a.reset(["g3"])
        assert e.value.kind == "tier_not_configured"
        rs.close()
    finally:
        a.close()
        b.close()


def test_vllm_connectors_pull_a_prefix_from_another_engine(hub, tmp_path):
    """Two scheduler-role vLLM connectors with ``remote_search.enabled``: engine A offloads a
    prompt to G2 (its G2 presence reaches the hub's indexer through the connector's event sink);
    engine B's GNMT stalls on the same prompt while its remote search opens a session on A's
    scheduler (A's pool exports come from the file its worker published) and hands the copy to
    B's workers as a pull op; once they report it, B registers the blocks and matches them."""
    import time
    from types import SimpleNamespace

    vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")
    from test_vllm_connector import _request, _sched_output, _vllm_config

    from kvbm_b200.connector import vllm_connector as vc
    from kvbm_b200.connector.protocol import ConnectorMetadata
    from kvbm_b200.connector.worker import run_remote_pull
    from kvbm_b200.engine.remote_search import pool_export

    def extra(iid):
        return {"leader": {"cache": {"host": {"num_blocks": 32}}, "hub": {"url": hub.url},
                           "remote_search": {"enabled": True, "timeout_secs": 5.0},
                           "events": {"policy": "all", "window_ms": 5},
                           "disagg": {"instance_id": iid, "directory": f"file://{tmp_path}"}}}

    Role = vllm_base.KVConnectorRole
    cfg = LayoutConfig.for_model(32, 2, 2, 64, BS)
    # each engine's worker: a G2 pool in a shared-memory file, published where its scheduler finds it
    pools = {}
    for iid in (701, 702):
        pools[iid] = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, location="shared")
        vc.g2_directory(SimpleNamespace(disagg=SimpleNamespace(directory=f"file://{tmp_path}"))).publish(
            iid, pool_export(pools[iid]), rank=0)
    a = vc.KvbmConnector(_vllm_config(extra(701)), Role.SCHEDULER)
    b = vc.KvbmConnector(_vllm_config(extra(702)), Role.SCHEDULER)
    try:
        tokens = list(range(3000, 3000 + 5 * BS + 3))
        ra = _request("a1", tokens)
        deadline = time.monotonic() + 5
        while (got := a.get_num_new_matched_tokens(ra, 0))[0] is None and time.monotonic() < deadline:
            time.sleep(0.01)  # A searches too (no other holder yet): a stall, then a cold miss
        assert got == (0, False)
        a.update_state_after_alloc(ra, SimpleNamespace(get_block_ids=lambda: ([0, 1, 2, 3, 4, 5],)), 0)
        m = ConnectorMetadata.decode(a.build_connector_meta(_sched_output([("a1", [0, 1, 2, 3, 4, 5])],
                                                                          {"a1": len(tokens)})).metadata)
        [off] = m.offload
        fill_blocks(pools[701], off.g2_ids, FillPattern.RANDOM, seed=4)  # what A's worker copied out of G1
        want = checksum_blocks(pools[701], off.g2_ids)
        a.update_connector_output(SimpleNamespace(finished_sending={"a1"}, finished_recving=None,
                                                  kv_connector_worker_meta=vc.KvbmConnectorWorkerMetadata(
                                                      {"offloaded": {m.step: 1}}), invalid_block_ids=set()))
        c = HubClient(hub.url)
        hashes = sequence_hashes(tokens, BS)
        deadline = time.monotonic() + 10
        while not c.query(hashes[:5]).get("hit") and time.monotonic() < deadline:
            time.sleep(0.01)  # A's presence events reach the indexer within an event window
        assert c.query(hashes[:5])["holders"] == [701]
        rb = _request("b1", tokens)
        n = None
        pull_meta = None
        while time.monotonic() < deadline:
            n, _ = b.get_num_new_matched_tokens(rb, 0)
            if n is not None:
                break
            # B's workers: run whatever pull the step's metadata carries and report it
            mb = ConnectorMetadata.decode(b.build_connector_meta(_sched_output([], {})).metadata)
            done = {}
            for op in mb.pull:
                run_remote_pull(op, pools[702], 0)
                done[op.pull_id] = 1
                pull_meta = op
            b.update_connector_output(SimpleNamespace(
                finished_sending=None, finished_recving=None, invalid_block_ids=set(),
                kv_connector_worker_meta=vc.KvbmConnectorWorkerMetadata({"pulled": done}) if done else None))
            time.sleep(0.01)
        assert n == 5 * BS, "B never matched the pulled prefix"
        assert pull_meta is not None and len(pull_meta.src_ids) == 5
        assert checksum_blocks(pools[702], pull_meta.g2_ids) == want  # same bytes in B's G2
        assert b._remote.search.stats["pulled_blocks"] == 5
        assert a._remote.holder.open_sessions() == 0  # A's session closed after the pull
    finally:
        a.shutdown()
        b.shutdown()
        for lay in pools.values():
            lay.backing.close()


def test_holder_stages_a_g3_continuation_before_the_pull(hub):
    """A holder whose prefix continues in G3 stages those blocks into G2 with its workers before
    answering, so the initiator pulls the whole match (2 blocks from G2 + 3 from G3)."""
    from kvbm_b200.physical.transfer import TransferCompleteNotification

    c = HubClient(hub.url)
    a = _Instance(801, c, KvBlockLayout.OPERATIONAL_NHD)
    b = _Instance(802, c, KvBlockLayout.OPERATIONAL_NHD)
    g3_layout = KvLayout.allocate(LayoutConfig.for_model(32, 2, 2, 64, BS), "fully_contiguous",
                                  KvBlockLayout.OPERATIONAL_NHD, location="shared")

    class StageWorker:  # moves G3 -> G2 bytes the way a worker's transfer manager does
        def execute_local_transfer(self, src_tier, src_ids, dst_tier, dst_ids, layer_range=None):
            assert (src_tier, dst_tier) == (Tier.G3, Tier.G2)
            a.layout.scatter_blocks(list(dst_ids), g3_layout.gather_blocks(list(src_ids)))
            return TransferCompleteNotification.ready()

    try:
        g3 = BlockManager(32, BS, "lru", Tier.G3, registry=a.g2.registry)
        a.leader.g3, a.leader.workers = g3, ParallelWorkers([StageWorker()])
        hashes = sequence_hashes(list(range(9000, 9000 + 5 * BS)), BS)
        hot = a.g2.allocate_blocks(2)
        fill_blocks(a.layout, [x.block_id for x in hot], FillPattern.RANDOM, seed=1)
        cold = g3.allocate_blocks(3)
        fill_blocks(g3_layout, [x.block_id for x in cold], FillPattern.RANDOM, seed=2)
        want = checksum_blocks(a.layout, [x.block_id for x in hot]) + checksum_blocks(g3_layout,
                                                                                       [x.block_id for x in cold])
        for x in a.g2.register_mutable(hot, hashes[:2]) + g3.register_mutable(cold, hashes[2:]):
            x.release()
        c.publish_events(a.iid, [("create", hashes)])
        rs = RemoteSearch(b.leader, [b.layout], b.msg, c, BS, RemoteSearchConfig(enabled=True))
        assert rs.pull(801, hashes) == 5
        got = b.g2.match_blocks(hashes)
        assert checksum_blocks(b.layout, [x.block_id for x in got]) == want
        assert a.g2.count_prefix(hashes) == 5  # the staged blocks stay in A's G2
        rs.close()
    finally:
        a.close()
        b.close()
        g3_layout.backing.close()
