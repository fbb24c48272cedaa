"""KV-event publishing: drain the registry's event queue in batches and ship
them to subscribers (the hub indexer over HTTP, a consolidator or router
over ZeroMQ PUB).

Batching follows the queue semantics (consecutive events of one kind,
creates ascending by position, removes descending, at most ``max_batch``
per batch); a publisher thread flushes every ``window_ms``. The wire message
carries the instance id so subscribers know whose cache changed.

Parity: crates/kvbm-logical/src/events/{manager.rs:169 (on_block_registered),
batcher.rs:22-78 (window 10 ms / max 1024), publisher.rs:170,
protocol.rs:56 (KvbmCacheEvents{events, instance_id})}.
"""

from __future__ import annotations

import threading
from typing import Callable

import msgpack
import zmq

from .. import _core_native as core


class EventsManager:
    def __init__(self, instance_id: int, policy: str = "power_of_two", min_position: int = 16,
                 max_position: int = 65536, window_ms: float = 10.0, max_batch: int = 1024):
        self.instance_id = instance_id
        self.queue = core.EventQueue(all_events=(policy == "all"), min_position=min_position,
                                     max_position=max_position)
        self.window_ms, self.max_batch = window_ms, max_batch
        self._sinks: list[Callable[[int, list[tuple[str, list[int]]]], None]] = []
        self._stop = threading.Event()
        self._t: threading.Thread | None = None
        self.published = 0

    def registry(self, frequency=None):
        """A block registry whose presence changes feed this manager's queue."""
        return core.Registry(events=self.queue, frequency=frequency)

    def add_sink(self, sink: Callable[[int, list[tuple[str, list[int]]]], None]) -> None:
        self._sinks.append(sink)

    def flush(self) -> list[tuple[str, list[int]]]:
        batches = self.queue.drain_batches(self.max_batch)
        if batches:
            for s in self._sinks:
                s(self.instance_id, batches)
            self.published += sum(len(b) for _, b in batches)
        return batches

    def start(self) -> "EventsManager":
        def run():
            while not self._stop.wait(self.window_ms / 1000.0):
                self.flush()
            self.flush()
        self._t = threading.Thread(target=run, daemon=True, name="kvbm-events")
        self._t.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)


class ZmqEventSink:
    """PUB socket sink: one message per flush, ``[instance_id, [[kind, [hashes...]], ...]]``."""

    def __init__(self, endpoint: str, topic: bytes = b"kvbm-events"):
        self.sock = zmq.Context.instance().socket(zmq.PUB)
        self.sock.setsockopt(zmq.LINGER, 0)
        if endpoint.endswith(":0"):
            port = self.sock.bind_to_random_port(endpoint[:-2])
            endpoint = f"{endpoint[:-2]}:{port}"
        else:
            self.sock.bind(endpoint)
        self.endpoint, self.topic = endpoint, topic

    def __call__(self, instance_id: int, batches) -> None:
        msg = [str(instance_id), [[k, [str(h) for h in hs]] for k, hs in batches]]
        self.sock.send_multipart([self.topic, msgpack.packb(msg, use_bin_type=True)])

    def close(self):
        self.sock.close(0)


class HubEventSink:
    """Posts batches to the hub indexer."""

    def __init__(self, client):
        self.client = client

    def __call__(self, instance_id: int, batches) -> None:
        self.client.publish_events(instance_id, batches)


def sink_for_endpoint(endpoint: str | None, hub_url: str | None = None):
    """The event sink an ``events.endpoint`` names: ``tcp://`` / ``ipc://`` binds a ZeroMQ PUB
    socket, ``nats://`` publishes on ``kvbm.events.<instance>`` through NATS, ``hub`` posts
    to the hub's indexer (``hub_url``); None names no sink."""
    if not endpoint:
        return None
    if endpoint.startswith(("tcp://", "ipc://", "inproc://")):
        return ZmqEventSink(endpoint)
    if endpoint.startswith("nats://"):
        from ..engine.pubsub import NatsPubSub, PubSubEventSink

        return PubSubEventSink(NatsPubSub(endpoint))
    if endpoint == "hub":
        if not hub_url:
            raise ValueError("events.endpoint = 'hub' needs hub.url")
        from ..hub.client import HubClient

        return HubEventSink(HubClient(hub_url))
    raise ValueError(f"unknown events endpoint {endpoint!r} (tcp://, ipc://, nats:// or hub)")


def events_from_config(cfg, instance_id: int, hub_url: str | None = None) -> EventsManager:
    """An EventsManager built from an ``EventsConfig``, its configured sink attached."""
    em = EventsManager(instance_id, policy=cfg.policy, min_position=cfg.min_position, max_position=cfg.max_position,
                       window_ms=cfg.window_ms, max_batch=cfg.max_batch)
    sink = sink_for_endpoint(cfg.endpoint, hub_url)
    if sink is not None:
        em.add_sink(sink)
    return em
