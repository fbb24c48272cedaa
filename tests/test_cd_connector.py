"""Conditional disaggregation through the connector, on CPU: the decode
leader's decision, dispatch and receive bookkeeping; the prefill leader's
push cursor over prefill chunks; the prefill plane and peer directory."""

import threading

import pytest
import torch.distributed as dist

from kvbm_b200.connector.leader import REMOTE_DECODE_KEY, ConnectorLeader, KvbmRequest, SchedulerOutputLite
from kvbm_b200.connector.protocol import ConnectorMetadata
from kvbm_b200.engine.cd import ConditionalDisagg, InflightBudget, SelectionPolicy
from kvbm_b200.engine.cd_plane import (LocalPeerDirectory, LocalPrefillPlane, StorePeerDirectory, StorePrefillPlane,
                                       decode_dispatch, encode_dispatch)
from kvbm_b200.engine.leader import InstanceLeader, ParallelWorkers
from kvbm_b200.logical.manager import BlockManager, Tier

BS = 16


def decode_leader(plane, slots=4, policy="always", budget=None, g2_blocks=64):
    g2 = BlockManager(g2_blocks, BS, "lineage", Tier.G2)
    cd = ConditionalDisagg(SelectionPolicy(policy, 64), InflightBudget(budget))
    return ConnectorLeader(InstanceLeader(g2, ParallelWorkers([])), BS, cd=cd, plane=plane, prefill_target=7,
                           instance_id=3, mailbox_slots=slots, recv_timeout_s=5.0)


def meta(leader, step, sched):
    return ConnectorMetadata.decode(leader.build_connector_meta(SchedulerOutputLite(step, sched)))


def test_decode_dispatches_and_receives():
    plane = LocalPrefillPlane()
    L = decode_leader(plane)
    prompt = list(range(100))  # 7 blocks (last one partial)
    L.create_slot(KvbmRequest("a", prompt))
    assert L.get_num_new_matched_tokens("a", 0) == (100, True)
    L.update_state_after_alloc("a", list(range(10, 18)), 100)
    [d] = plane.poll(7)
    assert d["request_id"] == "a" and list(d["tokens"]) == prompt
    dec = d["decode"]
    assert dec["instance"] == 3 and dec["dst_ids"] == list(range(10, 17)) and dec["provided_blocks"] == 0
    assert d["params"]["decode_endpoint"] == "3" and d["params"]["num_provided_tokens"] == 0
    m = meta(L, 1, {})
    assert len(m.recv) == 1 and m.recv[0].slot == dec["slot"] and m.recv[0].seq == dec["seq"]
    assert m.recv[0].g1_ids == list(range(10, 17))
    assert L.cd.budget.inflight == 1 and len(L._mailbox_free) == 3
    # vLLM asks again while the request waits: same answer, no second dispatch
    assert L.get_num_new_matched_tokens("a", 0) == (100, True)
    assert plane.poll(7) == []
    L.update_connector_output(finished_recving={"a"})
    assert L.cd.budget.inflight == 0 and len(L._mailbox_free) == 4
    assert L.cd_stats["received"] == 1
    assert L.request_finished("a") == (False, None)


def test_budget_and_mailbox_bound_remote_prefills():
    plane = LocalPrefillPlane()
    L = decode_leader(plane, slots=1)
    for rid in ("a", "b"):
        L.create_slot(KvbmRequest(rid, list(range(64))))
    assert L.get_num_new_matched_tokens("a", 0) == (64, True)
    assert L.get_num_new_matched_tokens("b", 0) == (0, False)  # no free mailbox slot: local prefill
    assert L.cd_stats == {**L.cd_stats, "remote": 1, "local": 1}
    assert L.cd.budget.inflight == 1


def test_threshold_policy_counts_connector_tokens():
    plane = LocalPrefillPlane()
    L = decode_leader(plane, policy="threshold")  # remote when >= 64 tokens still need prefill
    L.create_slot(KvbmRequest("short", list(range(40))))
    assert L.get_num_new_matched_tokens("short", 0) == (0, False)
    L.create_slot(KvbmRequest("long", list(range(1000, 1100))))
    assert L.get_num_new_matched_tokens("long", 0) == (100, True)


def test_g2_prefix_is_onboarded_and_rest_comes_remote():
    plane = LocalPrefillPlane()
    L = decode_leader(plane)
    L.cd = None  # warm G2 first with a local request
    prompt = list(range(100))
    L.create_slot(KvbmRequest("warm", prompt[:64] + [5]))
    L.update_state_after_alloc("warm", [0, 1, 2, 3, 4], 0)
    meta(L, 1, {"warm": ([], [], 65)})
    L.update_connector_output(worker_meta={"offloaded": {1: 1}})
    L.cd = ConditionalDisagg(SelectionPolicy("always"))
    L.create_slot(KvbmRequest("a", prompt))
    assert L.get_num_new_matched_tokens("a", 0) == (100, True)
    L.update_state_after_alloc("a", list(range(20, 28)), 100)
    m = meta(L, 2, {})
    assert [o.g1_ids for o in m.onboard] == [[20, 21, 22, 23]]
    [d] = plane.poll(7)
    assert d["decode"]["provided_blocks"] == 4 and d["decode"]["dst_ids"] == [24, 25, 26]
    assert d["params"]["num_provided_tokens"] == 64
    assert m.recv[0].g1_ids == [24, 25, 26]


def test_prefill_pushes_chunks_and_delays_free():
    g2 = BlockManager(8, BS, "lineage", Tier.G2)
    P = ConnectorLeader(InstanceLeader(g2, ParallelWorkers([])), BS, offload_enabled=False)
    prompt = list(range(100))
    remote = {"instance": 3, "dst_ids": list(range(40, 47)), "slot": 2, "seq": 11, "provided_blocks": 0}
    P.create_slot(KvbmRequest("a", prompt, kv_transfer_params={REMOTE_DECODE_KEY: remote}))
    assert P.get_num_new_matched_tokens("a", 0) == (0, False)
    P.update_state_after_alloc("a", list(range(7)), 0)
    m1 = meta(P, 1, {"a": ([], [], 48)})  # chunk 1: three complete blocks
    assert [(o.src_ids, o.dst_ids, o.final) for o in m1.push] == [([0, 1, 2], [40, 41, 42], False)]
    m2 = meta(P, 2, {"a": ([], [], 100)})  # last chunk: the rest, with the partial block
    [op] = m2.push
    assert op.src_ids == [3, 4, 5, 6] and op.dst_ids == [43, 44, 45, 46] and op.final
    assert (op.peer, op.slot, op.seq) == (3, 2, 11)
    assert P.request_finished("a") == (True, None)  # the push still reads its blocks
    P.update_connector_output(finished_sending={"a"})
    assert P.num_slots() == 0


def test_prefill_skips_blocks_the_decode_side_provides():
    g2 = BlockManager(8, BS, "lineage", Tier.G2)
    P = ConnectorLeader(InstanceLeader(g2, ParallelWorkers([])), BS, offload_enabled=False)
    remote = {"instance": 3, "dst_ids": [50, 51], "slot": 0, "seq": 1, "provided_blocks": 2}
    P.create_slot(KvbmRequest("a", list(range(64)), kv_transfer_params={REMOTE_DECODE_KEY: remote}))
    P.update_state_after_alloc("a", [0, 1, 2, 3], 0)
    [op] = meta(P, 1, {"a": ([], [], 64)}).push
    assert op.src_ids == [2, 3] and op.dst_ids == [50, 51] and op.final


def test_dispatch_wire_roundtrip():
    raw = encode_dispatch("r", [1, 2, 3], {"session_id": "s"}, {"instance": 1, "dst_ids": [4]}, salt="x")
    d = decode_dispatch(raw)
    assert d["request_id"] == "r" and d["tokens"].tolist() == [1, 2, 3] and d["decode"]["dst_ids"] == [4]
    assert d["salt"] == "x"


def test_store_plane_and_directory_in_order():
    store = dist.HashStore()
    plane = StorePrefillPlane(store)
    for i in range(3):
        plane.dispatch(5, encode_dispatch(f"r{i}", [i], {}, {}))
    plane.dispatch(6, encode_dispatch("other", [9], {}, {}))
    got = plane.poll(5, limit=2) + plane.poll(5)
    assert [d["request_id"] for d in got] == ["r0", "r1", "r2"]
    assert plane.poll(5) == []
    assert [d["request_id"] for d in plane.poll(6)] == ["other"]
    dirs = StorePeerDirectory(store)
    dirs.publish(5, {"mailbox": {"name": "m", "nbytes": 4096, "slots": 8}, "pool": {"x": b"\x01\x02"}})
    assert dirs.lookup(5, timeout_s=1)["pool"]["x"] == b"\x01\x02"


def test_local_plane_wait_wakes_on_dispatch():
    plane = LocalPrefillPlane()
    t = threading.Timer(0.05, lambda: plane.dispatch(1, encode_dispatch("late", [1], {}, {})))
    t.start()
    got = plane.wait(1, timeout_s=5.0)
    assert [d["request_id"] for d in got] == ["late"]
    d = LocalPeerDirectory()
    d.publish(1, {"a": 1})
    assert d.lookup(1)["a"] == 1


def test_decode_dispatch_routed_through_the_hub_to_a_prefill_server():
    """Decode leader -> hub prefill router -> PrefillRouterHandler -> prefill server's local plane;
    the router's call completes once the prefill engine finished the request."""
    from types import SimpleNamespace

    from kvbm_b200.engine.cd_plane import HubRouterPlane
    from kvbm_b200.hub.client import HubClient
    from kvbm_b200.hub.server import HubServer
    from kvbm_b200.runtime.messenger import wait_until
    from kvbm_b200.serving.prefill_server import PrefillServer

    class FakePrefill:
        role, instance_id = "prefill", 7

        def __init__(self):
            self.plane = LocalPrefillPlane()
            self.queue, self.seen = [], []
            self.engine = SimpleNamespace(has_unfinished=lambda: bool(self.queue), _delayed={})

        def pull(self, wait_s=0.0):
            got = self.plane.poll(self.instance_id)
            self.queue += got
            self.seen += got
            return len(got)

        def step(self):
            out = [SimpleNamespace(request_id=d["request_id"], num_prompt_tokens=int(d["tokens"].size))
                   for d in self.queue]
            self.queue = []
            return out

    hub = HubServer(max_seq_len=4096, ttl=5.0).start()
    fake = FakePrefill()
    server = PrefillServer(fake, hub.url)
    stop = threading.Event()
    t = threading.Thread(target=server.serve_forever, args=(stop,), daemon=True)
    t.start()
    client = HubClient(hub.url)
    plane = HubRouterPlane(client, timeout=10.0)
    try:
        assert wait_until(lambda: len(client.targets()) == 1, 5.0)
        L = decode_leader(plane)
        L.create_slot(KvbmRequest("routed", list(range(80))))
        assert L.get_num_new_matched_tokens("routed", 0) == (80, True)
        L.update_state_after_alloc("routed", list(range(30, 35)), 80)
        res = plane.futures[0].result(timeout=10)
        assert res["forwarded"] and res["result"]["result"]["request_id"] == "routed"
        [d] = fake.seen
        assert d["decode"]["dst_ids"] == list(range(30, 35)) and d["decode"]["instance"] == 3
    finally:
        stop.set()
        t.join(timeout=5)
        server.close()
        plane.close()
        hub.stop()


def test_engine_attached_to_the_prefill_router_serves_routed_prefills():
    """try_wrap_engine on a prefill-role engine config registers with the hub; a decode leader's
    dispatch routed by the hub becomes an engine.generate call carrying the decode instance in its
    kv_transfer_params; decode-role configs are not attached."""
    import asyncio
    from types import SimpleNamespace

    from kvbm_b200.engine.cd_plane import HubRouterPlane
    from kvbm_b200.hub.client import HubClient
    from kvbm_b200.hub.detect import connector_settings, try_wrap_engine
    from kvbm_b200.hub.server import HubServer
    from kvbm_b200.runtime.messenger import wait_until

    hub = HubServer(max_seq_len=4096, ttl=5.0).start()
    calls = []

    class FakeAsyncEngine:
        async def generate(self, prompt, params, request_id):
            calls.append((request_id, prompt["prompt_token_ids"], params))
            await asyncio.sleep(0.01)
            yield SimpleNamespace(finished=True)

    def cfg(extra):
        return SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_connector_extra_config=extra))

    assert connector_settings(cfg({"leader": {"hub": {"url": "u"}, "disagg": {"role": "prefill"}}})) == ("u", "prefill")
    loop = asyncio.new_event_loop()
    t = threading.Thread(target=loop.run_forever, daemon=True)
    t.start()
    client = HubClient(hub.url)
    plane = HubRouterPlane(client, timeout=10.0)
    handler = None
    try:
        assert try_wrap_engine(cfg({"hub": {"url": hub.url}, "disagg": {"role": "decode"}}), FakeAsyncEngine(),
                               loop) is None
        handler = try_wrap_engine(cfg({"hub": {"url": hub.url}, "disagg": {"role": "prefill"}}), FakeAsyncEngine(),
                                  loop, make_params=lambda n, p: {"max_tokens": n, "kv_transfer_params": p})
        assert handler is not None and wait_until(lambda: len(client.targets()) == 1, 5.0)
        L = decode_leader(plane)
        L.create_slot(KvbmRequest("vllm-routed", list(range(48))))
        assert L.get_num_new_matched_tokens("vllm-routed", 0) == (48, True)
        L.update_state_after_alloc("vllm-routed", [8, 9, 10], 48)
        res = plane.futures[0].result(timeout=10)
        assert res["forwarded"] and res["result"]["result"] == {"request_id": "vllm-routed", "finished": True}
        [(rid, toks, params)] = calls
        assert rid == "vllm-routed" and toks == list(range(48)) and params["max_tokens"] == 1
        ktp = params["kv_transfer_params"]
        assert ktp[REMOTE_DECODE_KEY]["dst_ids"] == [8, 9, 10] and ktp[REMOTE_DECODE_KEY]["instance"] == 3
    finally:
        if handler is not None:
            handler.close()
        plane.close()
        loop.call_soon_threadsafe(loop.stop)
        hub.stop()


def test_file_plane_serves_each_dispatch_once_across_pollers(tmp_path):
    """Several pollers of one prefill instance (e.g. threads of a prefill server) share the
    file plane's spool: every dispatch is served exactly once, in arrival order per poller."""
    from kvbm_b200.engine.cd_plane import FilePeerDirectory, FilePrefillPlane, encode_dispatch

    plane = FilePrefillPlane(str(tmp_path))
    for i in range(200):
        plane.dispatch(9, encode_dispatch(f"r{i}", [i], {}, {"instance": 1}))
    got: list[list[str]] = [[] for _ in range(4)]

    def poll(k):
        p = FilePrefillPlane(str(tmp_path))
        while True:
            batch = p.poll(9, limit=7)
            if not batch:
                return
            got[k] += [d["request_id"] for d in batch]

    ts = [threading.Thread(target=poll, args=(k,)) for k in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(10)
    served = sum(got, [])
    assert sorted(served, key=lambda r: int(r[1:])) == [f"r{i}" for i in range(200)]
    for g in got:
        assert g == sorted(g, key=lambda r: int(r[1:]))
    d = FilePeerDirectory(str(tmp_path))
    with pytest.raises(TimeoutError):
        d.lookup(5, timeout_s=0.05)
    d.publish(5, {"tp": 2}, rank=1)
    assert d.lookup(5, rank=1) == {"tp": 2}
    d.withdraw(5, rank=1)
    with pytest.raises(TimeoutError):
        d.lookup(5, timeout_s=0.05, rank=1)


def test_prefill_engine_served_from_the_file_plane_without_a_hub(tmp_path):
    """A prefill-role engine with a disaggregation instance id and no hub: try_wrap_engine serves
    the node's file plane, so a decode leader's dispatch becomes that engine's generate call
    carrying the decode instance in its kv_transfer_params."""
    import asyncio
    import time
    from types import SimpleNamespace

    from kvbm_b200.engine.cd_plane import FilePrefillPlane
    from kvbm_b200.hub.detect import PlaneServer, try_wrap_engine

    calls = []

    class FakeAsyncEngine:
        async def generate(self, prompt, params, request_id):
            calls.append((request_id, prompt["prompt_token_ids"], params))
            await asyncio.sleep(0.01)
            yield SimpleNamespace(finished=True)

    def cfg(disagg):
        return SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_connector_extra_config={"disagg": disagg}))

    loop = asyncio.new_event_loop()
    t = threading.Thread(target=loop.run_forever, daemon=True)
    t.start()
    url = f"file://{tmp_path}"
    server = None
    try:
        assert try_wrap_engine(cfg({"role": "prefill", "directory": url}), FakeAsyncEngine(), loop) is None  # no id
        server = try_wrap_engine(cfg({"role": "prefill", "instance_id": 7, "directory": url}), FakeAsyncEngine(),
                                 loop, make_params=lambda n, p: {"max_tokens": n, "kv_transfer_params": p})
        assert isinstance(server, PlaneServer)
        L = decode_leader(FilePrefillPlane(str(tmp_path)))
        L.create_slot(KvbmRequest("file-routed", list(range(40))))
        assert L.get_num_new_matched_tokens("file-routed", 0) == (40, True)
        L.update_state_after_alloc("file-routed", [4, 5, 6], 40)
        deadline = time.monotonic() + 10
        while not calls and time.monotonic() < deadline:
            time.sleep(0.01)
        [(rid, toks, params)] = calls
        assert rid == "file-routed" and toks == list(range(40)) and params["max_tokens"] == 1
        assert params["kv_transfer_params"][REMOTE_DECODE_KEY]["dst_ids"] == [4, 5, 6]
        assert server.served == 1
    finally:
        if server is not None:
            server.close()
        loop.call_soon_threadsafe(loop.stop)


def test_worker_withdraws_its_directory_entry_on_shutdown(tmp_path):
    """A connector worker that joined the plane removes its pool entry when it shuts down."""
    from kvbm_b200.connector.worker import ConnectorWorker
    from kvbm_b200.engine.cd_plane import FilePeerDirectory

    d = FilePeerDirectory(str(tmp_path))
    w = ConnectorWorker(device=0)
    w.instance_id, w.directory, w.tp_rank = 9, d, 0
    d.publish(9, {"tp": 1}, rank=0)
    assert d.lookup(9, timeout_s=0.1) == {"tp": 1}
    w.shutdown()
    with pytest.raises(TimeoutError):
        d.lookup(9, timeout_s=0.05)
