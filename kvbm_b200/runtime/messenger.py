"""Control-plane messaging: unary RPC handlers, distributed events and peer
discovery over ZeroMQ (TCP or IPC), msgpack-encoded.

Each process runs one :class:`Messenger` with a ROUTER socket served by a
background thread. Peers are addressed by instance id; the address book is
filled statically (``register_peer``) or from the hub. Handlers are plain
callables ``fn(payload) -> payload``. Distributed events are named one-shot
latches: any peer can ``trigger`` or ``poison`` an event, and a local
``wait_event`` returns once it fires (or raises if it was poisoned).

Parity: the reference's control plane is the external ``velo`` crate (TCP
active messages, typed unary handlers, distributed events used as completion
signals, hub-backed or static peer discovery; Cargo.toml:35-36,
crates/kvbm-engine/src/testing/messenger.rs:21-60) - same roles, own wire
format.
"""

from __future__ import annotations

import threading
import time
import uuid
from typing import Any, Callable

import msgpack
import zmq


class RpcError(RuntimeError):
    pass


class EventPoisoned(RuntimeError):
    pass


class _Event:
    __slots__ = ("flag", "poison")

    def __init__(self):
        self.flag = threading.Event()
        self.poison: str | None = None


class Messenger:
    def __init__(self, instance_id: int | None = None, bind: str = "tcp://127.0.0.1:0"):
        self.instance_id = instance_id if instance_id is not None else uuid.uuid4().int >> 64
        self.ctx = zmq.Context.instance()
        self._router = self.ctx.socket(zmq.ROUTER)
        self._router.setsockopt(zmq.LINGER, 0)
        if bind.startswith("tcp://") and bind.endswith(":0"):
            port = self._router.bind_to_random_port(bind[: -2])
            self.address = f"{bind[:-2]}:{port}"
        else:
            self._router.bind(bind)
            self.address = bind
        self._handlers: dict[str, Callable[[Any], Any]] = {}
        self._peers: dict[int, str] = {}
        self._events: dict[str, _Event] = {}
        self._ev_lock = threading.Lock()
        self._local = threading.local()
        self._stop = threading.Event()
        self.register_handler("_event.trigger", self._on_trigger)
        self.register_handler("_event.poison", self._on_poison)
        self.register_handler("_ping", lambda p: {"instance_id": self.instance_id})
        self._thread = threading.Thread(target=self._serve, name="kvbm-messenger", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------- server
    def register_handler(self, name: str, fn: Callable[[Any], Any]) -> None:
        self._handlers[name] = fn

    def _serve(self) -> None:
        poller = zmq.Poller()
        poller.register(self._router, zmq.POLLIN)
        while not self._stop.is_set():
            if not dict(poller.poll(50)):
                continue
            try:
                ident, _, raw = self._router.recv_multipart(zmq.NOBLOCK)
            except zmq.Again:
                continue
            try:
                msg = msgpack.unpackb(raw, raw=False)
                fn = self._handlers.get(msg["h"])
                if fn is None:
                    reply = {"ok": False, "err": f"no handler {msg['h']!r}"}
                else:
                    reply = {"ok": True, "r": fn(msg.get("p"))}
            except Exception as e:  # noqa: BLE001 - returned to the caller
                reply = {"ok": False, "err": f"{type(e).__name__}: {e}"}
            self._router.send_multipart([ident, b"", msgpack.packb(reply, use_bin_type=True)])

    # ------------------------------------------------------------- client
    def register_peer(self, instance_id: int, address: str) -> None:
        self._peers[int(instance_id)] = address

    def peer_info(self) -> dict:
        return {"instance_id": self.instance_id, "address": self.address}

    def _sock(self, address: str):
        socks = getattr(self._local, "socks", None)
        if socks is None:
            socks = self._local.socks = {}
        s = socks.get(address)
        if s is None:
            s = self.ctx.socket(zmq.DEALER)
            s.setsockopt(zmq.LINGER, 0)
            s.connect(address)
            socks[address] = s
        return s

    def call(self, peer: int | str, handler: str, payload: Any = None, timeout: float = 30.0) -> Any:
        address = peer if isinstance(peer, str) else self._peers.get(int(peer))
        if address is None:
            raise RpcError(f"unknown peer {peer}")
        s = self._sock(address)
        s.send_multipart([b"", msgpack.packb({"h": handler, "p": payload}, use_bin_type=True)])
        if not s.poll(int(timeout * 1000)):
            # the socket may hold a late reply: drop it so the next call is not confused
            s.close(0)
            self._local.socks.pop(address, None)
            raise TimeoutError(f"rpc {handler!r} to {peer} timed out after {timeout}s")
        _, raw = s.recv_multipart()
        reply = msgpack.unpackb(raw, raw=False)
        if not reply["ok"]:
            raise RpcError(reply["err"])
        return reply.get("r")

    # ------------------------------------------------------------- events
    def new_event(self, name: str | None = None) -> str:
        name = name or f"{self.instance_id}:{uuid.uuid4().hex}"
        with self._ev_lock:
            self._events.setdefault(name, _Event())
        return name

    def _ev(self, name: str) -> _Event:
        with self._ev_lock:
            return self._events.setdefault(name, _Event())

    def _on_trigger(self, name):
        self._ev(name).flag.set()
        return True

    def _on_poison(self, p):
        ev = self._ev(p["name"])
        ev.poison = p.get("reason", "poisoned")
        ev.flag.set()
        return True

    def trigger(self, name: str, owner: int | None = None) -> None:
        if owner is None or owner == self.instance_id:
            self._on_trigger(name)
        else:
            self.call(owner, "_event.trigger", name)

    def poison(self, name: str, reason: str, owner: int | None = None) -> None:
        if owner is None or owner == self.instance_id:
            self._on_poison({"name": name, "reason": reason})
        else:
            self.call(owner, "_event.poison", {"name": name, "reason": reason})

    def wait_event(self, name: str, timeout: float | None = None) -> None:
        ev = self._ev(name)
        if not ev.flag.wait(timeout):
            raise TimeoutError(f"event {name} not triggered within {timeout}s")
        if ev.poison is not None:
            raise EventPoisoned(ev.poison)

    def is_triggered(self, name: str) -> bool:
        return self._ev(name).flag.is_set()

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2)
        self._router.close(0)


class MessengerPair:
    """Two messengers on loopback that know each other (tests, in-process pairs)."""

    def __init__(self):
        self.a = Messenger()
        self.b = Messenger()
        self.a.register_peer(self.b.instance_id, self.b.address)
        self.b.register_peer(self.a.instance_id, self.a.address)

    def close(self):
        self.a.close()
        self.b.close()


def wait_until(pred: Callable[[], bool], timeout: float, poll: float = 0.01) -> bool:
    deadline = time.monotonic() + timeout
    while time.monotonic() < deadline:
        if pred():
            return True
        time.sleep(poll)
    return pred()
