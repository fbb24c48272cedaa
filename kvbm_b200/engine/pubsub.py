"""Subject-based publish/subscribe for engine events.

One interface, three transports:

* :class:`StubPubSub` - in-process (tests, single-process deployments);
* :class:`ZmqPubSub` - ZeroMQ PUB/SUB; ``connect`` another endpoint to
  receive its subjects (subjects are ZeroMQ topic prefixes);
* :class:`NatsPubSub` - a NATS server, through a client of the NATS text
  protocol written here (``PUB`` / ``SUB`` / ``MSG`` / ``PING`` over TCP), so
  no client package is needed.

``make_pubsub(url)`` picks the transport from the URL scheme (``stub://``,
``tcp://`` / ``ipc://``, ``nats://``). :class:`PubSubEventSink` plugs a
transport into ``logical.events.EventsManager``.

Parity: crates/kvbm-engine/src/pubsub/{mod.rs (Publisher/Subscriber
traits), stub.rs, nats.rs}.
"""

from __future__ import annotations

import threading
from collections import defaultdict
from typing import Callable

import msgpack
import zmq

Handler = Callable[[str, bytes], None]


class PubSub:
    def publish(self, subject: str, payload: bytes) -> None:
        raise NotImplementedError

    def subscribe(self, subject: str, handler: Handler) -> None:
        raise NotImplementedError

    def close(self) -> None:
        pass


class StubPubSub(PubSub):
    """Delivers synchronously to handlers whose subject is a prefix of the published one."""

    def __init__(self):
        self._subs: dict[str, list[Handler]] = defaultdict(list)
        self._lock = threading.Lock()
        self.published = 0

    def publish(self, subject: str, payload: bytes) -> None:
        with self._lock:
            targets = [h for s, hs in self._subs.items() if subject.startswith(s) for h in hs]
            self.published += 1
        for h in targets:
            h(subject, payload)

    def subscribe(self, subject: str, handler: Handler) -> None:
        with self._lock:
            self._subs[subject].append(handler)


class ZmqPubSub(PubSub):
    """PUB socket bound at ``bind``; SUB socket connected to any number of peers."""

    def __init__(self, bind: str = "tcp://127.0.0.1:0"):
        self.ctx = zmq.Context.instance()
        self._pub = self.ctx.socket(zmq.PUB)
        self._pub.setsockopt(zmq.LINGER, 0)
        self._pub.bind(bind)
        self.endpoint = self._pub.getsockopt_string(zmq.LAST_ENDPOINT)
        self._sub = self.ctx.socket(zmq.SUB)
        self._sub.setsockopt(zmq.LINGER, 0)
        self._handlers: dict[str, list[Handler]] = defaultdict(list)
        self._pub_lock = threading.Lock()
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._loop, daemon=True, name="kvbm-pubsub")
        self._sub_lock = threading.Lock()
        self._pending: list[tuple[str, str]] = []  # (op, arg) applied by the receive thread
        self._t.start()

    def connect(self, endpoint: str) -> None:
        with self._sub_lock:
            self._pending.append(("connect", endpoint))

    def publish(self, subject: str, payload: bytes) -> None:
        with self._pub_lock:
            self._pub.send_multipart([subject.encode(), payload])

    def subscribe(self, subject: str, handler: Handler) -> None:
        with self._sub_lock:
            self._handlers[subject].append(handler)
            self._pending.append(("subscribe", subject))

    def _loop(self) -> None:
        poller = zmq.Poller()
        poller.register(self._sub, zmq.POLLIN)
        while not self._stop.is_set():
            with self._sub_lock:
                ops, self._pending = self._pending, []
            for op, arg in ops:  # zmq sockets are used from this thread only
                if op == "connect":
                    self._sub.connect(arg)
                else:
                    self._sub.setsockopt(zmq.SUBSCRIBE, arg.encode())
            if not dict(poller.poll(20)):
                continue
            subject, payload = self._sub.recv_multipart()
            s = subject.decode()
            with self._sub_lock:
                targets = [h for k, hs in self._handlers.items() if s.startswith(k) for h in hs]
            for h in targets:
                h(s, payload)

    def close(self) -> None:
        self._stop.set()
        self._t.join(timeout=2)
        self._sub.close(0)
        self._pub.close(0)


class NatsPubSub(PubSub):
    """A NATS client speaking the NATS client protocol directly over TCP (no client package).

    Connects to ``nats://[user:pass@]host[:port]`` (port 4222 by default),
    reads the server's ``INFO``, sends ``CONNECT`` (and the credentials in
    the URL) and waits for the ``PONG`` of a ``PING`` before returning, so a
    refused connection fails here. ``publish`` writes one ``PUB``; a reader
    thread answers the server's ``PING`` and delivers every ``MSG`` to the
    handler of its subscription. Subjects get ``prefix.`` in front when a
    prefix is set. ``subscribe`` follows the other transports' prefix
    semantics: a subject without wildcards receives itself and every subject
    below it (``a.b`` and ``a.b.>``); a subject with NATS wildcards (``*``,
    ``>``) is passed to the server as is. ``flush`` waits until the server
    has processed everything sent before it (a ``PING`` / ``PONG`` round
    trip). A server ``-ERR`` is kept in ``last_error`` and raised by the
    next ``flush``.
    """

    def __init__(self, url: str, prefix: str | None = None, name: str = "kvbm", timeout: float = 5.0):
        import json
        import socket
        from urllib.parse import urlparse

        u = urlparse(url)
        if u.scheme != "nats":
            raise ValueError(f"not a nats:// URL: {url!r}")
        self.prefix = prefix.rstrip(".") if prefix else None
        self.timeout = timeout
        self._sock = socket.create_connection((u.hostname or "127.0.0.1", u.port or 4222), timeout=timeout)
        self._rfile = self._sock.makefile("rb")
        line = self._rfile.readline()
        if not line.startswith(b"INFO "):
            raise ConnectionError(f"not a NATS server (first line {line[:40]!r})")
        self.server_info = json.loads(line[5:])
        opts = {"verbose": False, "pedantic": False, "name": name, "lang": "python", "version": "kvbm-b200",
                "protocol": 1, "headers": False}
        if u.username:
            opts.update(user=u.username, **({"pass": u.password} if u.password is not None else {}))
        self._wlock = threading.Lock()
        self._handlers: dict[int, tuple[str, Handler]] = {}
        self._sid = 0
        self._pongs = 0
        self._pings_sent = 0
        self._cv = threading.Condition()
        self.last_error: str | None = None
        self._closed = False
        self._send(b"CONNECT " + json.dumps(opts).encode() + b"\r\n")
        self._sock.settimeout(None)
        self._t = threading.Thread(target=self._read_loop, daemon=True, name="kvbm-nats")
        self._t.start()
        self.flush(timeout)

    def _subject(self, subject: str) -> str:
        return f"{self.prefix}.{subject}" if self.prefix else subject

    def _send(self, data: bytes) -> None:
        with self._wlock:
            self._sock.sendall(data)

    def _read_loop(self) -> None:
        f = self._rfile
        try:
            while True:
                line = f.readline()
                if not line:
                    break
                if line.startswith(b"MSG "):
                    parts = line[4:].split()
                    subject, sid, size = parts[0].decode(), int(parts[1]), int(parts[-1])
                    payload = f.read(size + 2)[:size]
                    h = self._handlers.get(sid)
                    if h is not None:
                        h[1](subject[len(self.prefix) + 1:] if self.prefix and subject.startswith(self.prefix + ".")
                             else subject, payload)
                elif line.startswith(b"PING"):
                    self._send(b"PONG\r\n")
                elif line.startswith(b"PONG"):
                    with self._cv:
                        self._pongs += 1
                        self._cv.notify_all()
                elif line.startswith(b"-ERR"):
                    with self._cv:
                        self.last_error = line[4:].strip().decode(errors="replace")
                        self._cv.notify_all()
                # +OK and INFO updates need no action
        except (OSError, ValueError):
            pass
        finally:
            with self._cv:
                self._closed = True
                self._cv.notify_all()

    def publish(self, subject: str, payload: bytes) -> None:
        subj = self._subject(subject).encode()
        self._send(b"PUB " + subj + b" " + str(len(payload)).encode() + b"\r\n" + bytes(payload) + b"\r\n")

    def subscribe(self, subject: str, handler: Handler) -> None:
        subj = self._subject(subject)
        patterns = [subj] if ("*" in subj.split(".") or subj.endswith(">")) else [subj, subj + ".>"]
        for pat in patterns:
            with self._wlock:
                self._sid += 1
                sid = self._sid
            self._handlers[sid] = (pat, handler)
            self._send(f"SUB {pat} {sid}\r\n".encode())

    def flush(self, timeout: float | None = None) -> None:
        """Wait until the server has processed everything sent so far."""
        with self._cv:
            self._pings_sent += 1
            want = self._pings_sent
        self._send(b"PING\r\n")
        with self._cv:
            ok = self._cv.wait_for(lambda: self._pongs >= want or self.last_error is not None or self._closed,
                                   timeout=timeout if timeout is not None else self.timeout)
            if self.last_error is not None:
                err, self.last_error = self.last_error, None
                raise ConnectionError(f"NATS server error: {err}")
            if self._closed:
                raise ConnectionError("NATS connection closed")
            if not ok:
                raise TimeoutError("NATS server did not answer PING")

    def close(self) -> None:
        import socket

        try:
            self._sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self._sock.close()
        self._t.join(timeout=2)


def make_pubsub(url: str) -> PubSub:
    if url.startswith("stub://"):
        return StubPubSub()
    if url.startswith(("tcp://", "ipc://", "inproc://")):
        return ZmqPubSub(url)
    if url.startswith("nats://"):
        return NatsPubSub(url)  # NATS subjects: '.'-separated tokens
    raise ValueError(f"no pub/sub transport for {url!r}")


class PubSubEventSink:
    """``EventsManager`` sink: one msgpack message per flush on ``<prefix>.<instance>``."""

    def __init__(self, pubsub: PubSub, prefix: str = "kvbm.events"):
        self.pubsub, self.prefix = pubsub, prefix

    def __call__(self, instance_id: int, batches: list[tuple[str, list[int]]]) -> None:
        body = msgpack.packb({"instance_id": str(instance_id),
                              "batches": [[k, [str(h) for h in hs]] for k, hs in batches]}, use_bin_type=True)
        self.pubsub.publish(f"{self.prefix}.{instance_id}", body)

    @staticmethod
    def decode(payload: bytes) -> tuple[int, list[tuple[str, list[int]]]]:
        d = msgpack.unpackb(payload, raw=False)
        return int(d["instance_id"]), [(k, [int(h) for h in hs]) for k, hs in d["batches"]]
