"""Subject-based publish/subscribe for engine events.

One interface, three transports:

* :class:`StubPubSub` - in-process (tests, single-process deployments);
* :class:`ZmqPubSub` - ZeroMQ PUB/SUB; ``connect`` another endpoint to
  receive its subjects (subjects are ZeroMQ topic prefixes);
* :class:`NatsPubSub` - a NATS server, when the ``nats`` client package is
  installed (it is optional and not bundled; constructing one without it
  raises ``ImportError``).

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


class NatsPubSub(PubSub):  # pragma: no cover - needs the optional nats client and a server
    def __init__(self, url: str):
        try:
            import nats  # noqa: F401
        except ImportError as e:
            raise ImportError("NatsPubSub needs the optional 'nats-py' package") from e
        import asyncio

        self._loop = asyncio.new_event_loop()
        self._t = threading.Thread(target=self._loop.run_forever, daemon=True, name="kvbm-nats")
        self._t.start()
        self._nc = asyncio.run_coroutine_threadsafe(nats.connect(url), self._loop).result(10)

    def publish(self, subject: str, payload: bytes) -> None:
        import asyncio

        asyncio.run_coroutine_threadsafe(self._nc.publish(subject, payload), self._loop).result(10)

    def subscribe(self, subject: str, handler: Handler) -> None:
        import asyncio

        async def cb(msg):
            handler(msg.subject, msg.data)

        asyncio.run_coroutine_threadsafe(self._nc.subscribe(subject + ">", cb=cb), self._loop).result(10)

    def close(self) -> None:
        import asyncio

        asyncio.run_coroutine_threadsafe(self._nc.close(), self._loop).result(10)
        self._loop.call_soon_threadsafe(self._loop.stop)


def make_pubsub(url: str) -> PubSub:
    if url.startswith("stub://"):
        return StubPubSub()
    if url.startswith(("tcp://", "ipc://", "inproc://")):
        return ZmqPubSub(url)
    if url.startswith("nats://"):
        return NatsPubSub(url)
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
