"""The NATS pub/sub transport against an in-process server that speaks the NATS client
protocol (INFO / CONNECT / PUB / SUB / UNSUB / MSG / PING / PONG, ``*`` and ``>``
subject wildcards, user/password check), on CPU."""

import json
import socket
import threading
import time

import pytest

from kvbm_b200.engine.pubsub import NatsPubSub, PubSubEventSink, make_pubsub


def _matches(pattern: str, subject: str) -> bool:
    p, s = pattern.split("."), subject.split(".")
    for i, tok in enumerate(p):
        if tok == ">":
            return len(s) > i
        if i >= len(s) or (tok != "*" and tok != s[i]):
            return False
    return len(p) == len(s)


class MiniNatsServer:
    """Enough of a NATS server for one test: routes PUB to matching SUBs of every client."""

    def __init__(self, user=None, password=None):
        self.user, self.password = user, password
        self.srv = socket.socket()
        self.srv.bind(("127.0.0.1", 0))
        self.srv.listen()
        self.port = self.srv.getsockname()[1]
        self.subs = []  # (conn, wfile lock, sid, pattern)
        self.lock = threading.Lock()
        self.published = 0
        threading.Thread(target=self._accept, daemon=True).start()

    def _accept(self):
        while True:
            try:
                c, _ = self.srv.accept()
            except OSError:
                return
            threading.Thread(target=self._serve, args=(c,), daemon=True).start()

    def _serve(self, c):
        wl = threading.Lock()

        def send(b):
            with wl:
                c.sendall(b)

        send(b"INFO " + json.dumps({"server_id": "mini", "version": "2.10.0", "max_payload": 1 << 20}).encode()
             + b"\r\n")
        f = c.makefile("rb")
        try:
            while True:
                line = f.readline()
                if not line:
                    return
                op = line.split(b" ", 1)[0].strip().upper()
                if op == b"CONNECT":
                    opts = json.loads(line[8:])
                    if self.user is not None and (opts.get("user"), opts.get("pass")) != (self.user, self.password):
                        send(b"-ERR 'Authorization Violation'\r\n")
                        c.close()
                        return
                elif op == b"PING":
                    send(b"PONG\r\n")
                elif op == b"SUB":
                    _, subj, sid = line.split()
                    with self.lock:
                        self.subs.append((c, send, sid, subj.decode()))
                elif op == b"UNSUB":
                    sid = line.split()[1]
                    with self.lock:
                        self.subs = [x for x in self.subs if not (x[0] is c and x[2] == sid)]
                elif op == b"PUB":
                    parts = line.split()
                    subj, n = parts[1].decode(), int(parts[-1])
                    payload = f.read(n + 2)[:n]
                    with self.lock:
                        self.published += 1
                        targets = [(snd, sid) for (_, snd, sid, pat) in self.subs if _matches(pat, subj)]
                    for snd, sid in targets:
                        snd(b"MSG " + subj.encode() + b" " + sid + b" " + str(n).encode() + b"\r\n" + payload + b"\r\n")
        except OSError:
            return

    def url(self, creds=""):
        return f"nats://{creds}127.0.0.1:{self.port}"

    def close(self):
        self.srv.close()


@pytest.fixture
def server():
    s = MiniNatsServer()
    yield s
    s.close()


def _collect():
    got, ev = [], threading.Event()

    def h(subject, payload):
        got.append((subject, payload))
        ev.set()
    return got, ev, h


def test_publish_subscribe_prefix_and_wildcards(server):
    a, b = NatsPubSub(server.url()), make_pubsub(server.url())
    try:
        assert a.server_info["server_id"] == "mini"
        got, _, h = _collect()
        b.subscribe("kvbm.events", h)           # prefix semantics: the subject and everything below it
        wild, _, hw = _collect()
        b.subscribe("kvbm.*.g2", hw)            # a NATS wildcard goes to the server as is
        b.flush()
        a.publish("kvbm.events", b"root")
        a.publish("kvbm.events.17", b"x" * 70000)  # larger than one socket read
        a.publish("kvbm.eventsX.1", b"no")      # not below the subject (token boundary)
        a.publish("kvbm.blocks.g2", b"w")
        a.flush()
        deadline = time.monotonic() + 5
        while (len(got) < 2 or not wild) and time.monotonic() < deadline:
            time.sleep(0.01)
        assert sorted(s for s, _ in got) == ["kvbm.events", "kvbm.events.17"]
        assert dict(got)["kvbm.events.17"] == b"x" * 70000
        assert wild == [("kvbm.blocks.g2", b"w")]
    finally:
        a.close()
        b.close()


def test_subject_prefix_and_event_sink(server):
    pub = NatsPubSub(server.url(), prefix="tenant")
    sub = NatsPubSub(server.url(), prefix="tenant")
    raw = NatsPubSub(server.url())
    try:
        got, ev, h = _collect()
        sub.subscribe("kvbm.events", h)
        seen, ev2, h2 = _collect()
        raw.subscribe("tenant.kvbm.events", h2)  # what actually travels carries the prefix
        sub.flush()
        raw.flush()
        PubSubEventSink(pub)(42, [("create", [1, 2]), ("remove", [3])])
        pub.flush()
        assert ev.wait(5) and ev2.wait(5)
        subject, payload = got[0]
        assert subject == "kvbm.events.42" and seen[0][0] == "tenant.kvbm.events.42"
        assert PubSubEventSink.decode(payload) == (42, [("create", [1, 2]), ("remove", [3])])
    finally:
        for c in (pub, sub, raw):
            c.close()


def test_credentials_and_refused_connection():
    s = MiniNatsServer(user="kv", password="bm")
    try:
        ok = NatsPubSub(s.url("kv:bm@"))
        ok.close()
        with pytest.raises(ConnectionError):
            NatsPubSub(s.url("kv:wrong@"), timeout=2)
    finally:
        s.close()
    with pytest.raises(OSError):
        NatsPubSub(s.url(), timeout=1)  # nothing listens any more
    with pytest.raises(ValueError):
        NatsPubSub("tcp://127.0.0.1:1")


def test_connector_publishes_g2_events_through_nats(server):
    """A scheduler-role vLLM connector with ``events.enabled`` and a ``nats://`` endpoint: once a
    request's offloaded blocks are registered in G2, their presence events reach a NATS subscriber."""
    from types import SimpleNamespace

    pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")
    from test_vllm_connector import _request, _sched_output, _vllm_config, vllm_base  # noqa: E402

    from kvbm_b200.connector import vllm_connector as vc
    from kvbm_b200.engine.pubsub import PubSubEventSink

    sub = NatsPubSub(server.url())
    got, ev, h = _collect()
    sub.subscribe("kvbm.events", h)
    sub.flush()
    conn = vc.KvbmConnector(_vllm_config({"leader": {"cache": {"host": {"num_blocks": 64}},
                                                     "events": {"enabled": True, "endpoint": server.url(),
                                                                "policy": "all", "window_ms": 5}}}),
                            vllm_base.KVConnectorRole.SCHEDULER)
    try:
        tokens = list(range(5 * 16 + 3))
        r = _request("a", tokens)
        conn.get_num_new_matched_tokens(r, 0)
        conn.update_state_after_alloc(r, SimpleNamespace(get_block_ids=lambda: ([10, 11, 12, 13, 14, 15],)), 0)
        conn.build_connector_meta(_sched_output([("a", [10, 11, 12, 13, 14, 15])], {"a": len(tokens)}))
        wm = vc.KvbmConnectorWorkerMetadata({"offloaded": {1: 1}})
        conn.update_connector_output(SimpleNamespace(finished_sending={"a"}, finished_recving=None,
                                                     kv_connector_worker_meta=wm, invalid_block_ids=set()))
        assert ev.wait(5)
        iid, batches = PubSubEventSink.decode(got[0][1])
        created = [h for kind, hs in batches if kind == "create" for h in hs]
        assert len(created) == 5  # the five full prompt blocks became present in G2
    finally:
        conn.shutdown()
        sub.close()
