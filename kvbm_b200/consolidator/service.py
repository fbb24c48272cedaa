"""KV-event consolidator: one deduplicated event stream for a KV-aware router.

Ingress:
* the serving engine's own G1 events over ZeroMQ SUB (vLLM / TRT-LLM
  ``KvEventBatch`` msgpack payloads, 2-frame ``[topic, payload]`` or 3-frame
  ``[topic, seq, payload]``): ``BlockStored`` (token ids chunked by block
  size, parents chained left to right), ``BlockRemoved``,
  ``AllBlocksCleared``;
* the block manager's own events (G2/G3 presence from the registry's event
  queue), which carry sequence hashes but no tokens.

Everything goes through the native :class:`ConsolidatorTracker` (first STORE
publishes, last REMOVE publishes, KVBM-only blocks wait for a token-carrying
source). Egress is a ZeroMQ PUB socket in the router's msgpack wire format:
``[timestamp, [events...], data_parallel_rank]`` with ``BlockStored`` /
``BlockRemoved`` / ``AllBlocksCleared`` maps; 128-bit sequence hashes are
projected to the router's u64 hash (the lineage word).

Parity: crates/kvbm-consolidator/src/{lib.rs, tracker.rs, hash.rs (128->64
projection), ingress/zmq_subscriber.rs, ingress/kvbm_bridge.rs,
egress/zmq_publisher.rs, wire/router_out.rs, wire/vllm_in.rs}.
"""

from __future__ import annotations

import threading
import time

import msgpack
import zmq

from .. import _core_native as core

SOURCES = {"vllm": 0, "gpu": 0, "trtllm": 1, "tensorrt-llm": 1, "kvbm": 2}


def source_id(name: str) -> int:
    try:
        return SOURCES[name.lower()]
    except KeyError:
        raise ValueError(f"Unknown event source: {name}") from None


class Consolidator:
    def __init__(self, publish_endpoint: str | None = None, block_size: int = 16, dp_rank: int | None = None):
        self.tracker = core.ConsolidatorTracker()
        self.block_size = block_size
        self.dp_rank = dp_rank
        self.ctx = zmq.Context.instance()
        self.pub = None
        if publish_endpoint:
            self.pub = self.ctx.socket(zmq.PUB)
            self.pub.setsockopt(zmq.LINGER, 0)
            if publish_endpoint.endswith(":0"):
                port = self.pub.bind_to_random_port(publish_endpoint[:-2])
                publish_endpoint = f"{publish_endpoint[:-2]}:{port}"
            else:
                self.pub.bind(publish_endpoint)
        self.endpoint = publish_endpoint
        self._lock = threading.Lock()
        self._threads: list[threading.Thread] = []
        self._stop = threading.Event()
        self.stats = {"in_batches": 0, "bad_batches": 0, "out_batches": 0}

    # ---------------------------------------------------------- ingress
    def ingest_engine_batch(self, payload: bytes, source: str = "vllm") -> None:
        """Apply one msgpack KvEventBatch from an engine (vLLM / TRT-LLM)."""
        try:
            batch = msgpack.unpackb(payload, raw=False, strict_map_key=False)
        except Exception:  # noqa: BLE001 - malformed input must not kill the loop
            self.stats["bad_batches"] += 1
            return
        events = batch[1] if isinstance(batch, (list, tuple)) else batch.get("events", [])
        src = source_id(source)
        with self._lock:
            self.stats["in_batches"] += 1
            for ev in events:
                kind, body = _event_kind(ev)
                if kind == "BlockStored":
                    hashes = [str(h) for h in body.get("block_hashes", [])]
                    parent = body.get("parent_block_hash")
                    parent = None if parent is None else str(parent)
                    toks = list(body.get("token_ids", []))
                    bs = int(body.get("block_size", self.block_size))
                    lora = body.get("lora_name") or ""
                    for i, h in enumerate(hashes):
                        chunk = toks[i * bs:(i + 1) * bs]
                        self.tracker.handle_store(src, h, parent, chunk, bs, lora)
                        parent = h
                elif kind == "BlockRemoved":
                    for h in body.get("block_hashes", []):
                        self.tracker.handle_remove(src, str(h))
                elif kind == "AllBlocksCleared":
                    self.tracker.handle_clear_all()

    def ingest_kvbm_events(self, events: list[tuple[str, int]]) -> None:
        """Apply (kind, seq_hash) pairs drained from the block manager's event queue."""
        with self._lock:
            for kind, h in events:
                if kind == "create":
                    self.tracker.handle_kvbm_store(h)
                else:
                    self.tracker.handle_kvbm_remove(h)

    # ----------------------------------------------------------- egress
    def flush(self) -> list[dict]:
        with self._lock:
            evs = self.tracker.drain_events()
        if not evs:
            return []
        out = []
        for e in evs:
            if e["kind"] == "store":
                h = e["seq_hash"]
                parent = (h >> 64) & ((1 << 64) - 1)
                d = {"type": "BlockStored", "block_hashes": [e["router_hash"]],
                     "parent_block_hash": parent if parent else None, "token_ids": e["token_ids"],
                     "block_size": e["block_size"]}
                if e.get("lora_name"):
                    d["lora_name"] = e["lora_name"]
            elif e["kind"] == "remove":
                d = {"type": "BlockRemoved", "block_hashes": [e["router_hash"]]}
            else:
                d = {"type": "AllBlocksCleared"}
            out.append(d)
        if self.pub is not None:
            self.pub.send_multipart([b"kv-events", msgpack.packb([time.time(), out, self.dp_rank],
                                                                 use_bin_type=True)])
            self.stats["out_batches"] += 1
        return out

    def subscribe(self, endpoint: str, source: str = "vllm", topic: bytes = b"") -> None:
        """Start a SUB loop on an engine's event endpoint."""
        sock = self.ctx.socket(zmq.SUB)
        sock.setsockopt(zmq.LINGER, 0)
        sock.setsockopt(zmq.SUBSCRIBE, topic)
        sock.connect(endpoint)

        def loop():
            poller = zmq.Poller()
            poller.register(sock, zmq.POLLIN)
            while not self._stop.is_set():
                if not dict(poller.poll(50)):
                    continue
                frames = sock.recv_multipart()
                if len(frames) not in (2, 3):
                    self.stats["bad_batches"] += 1
                    continue
                self.ingest_engine_batch(frames[-1], source)
                self.flush()
            sock.close(0)

        t = threading.Thread(target=loop, daemon=True, name="kvbm-consolidator-sub")
        t.start()
        self._threads.append(t)

    def close(self) -> None:
        self._stop.set()
        for t in self._threads:
            t.join(timeout=2)
        if self.pub is not None:
            self.pub.close(0)


def _event_kind(ev):
    """vLLM encodes events either as tagged maps or as [tag, ...fields] arrays."""
    if isinstance(ev, dict):
        return ev.get("type") or ev.get("kind"), ev
    if isinstance(ev, (list, tuple)) and ev:
        tag = ev[0]
        if tag == "BlockStored":
            keys = ["block_hashes", "parent_block_hash", "token_ids", "block_size", "lora_id", "medium"]
            return tag, dict(zip(keys, ev[1:]))
        if tag == "BlockRemoved":
            return tag, dict(zip(["block_hashes", "medium"], ev[1:]))
        return tag, {}
    return None, {}


def start_leader_consolidator(vllm_endpoint: str | None, output_bind: str, source: str = "vllm",
                              block_size: int = 16, events=None) -> Consolidator:
    """The consolidator a scheduler-side connector runs: subscribed to the engine's KV-event
    endpoint, publishing on ``output_bind``, and fed the block manager's own G2/G3 presence
    events when ``events`` (a ``logical.events.EventsManager``) is given."""
    c = Consolidator(publish_endpoint=output_bind, block_size=block_size)
    if vllm_endpoint:
        c.subscribe(vllm_endpoint, source=source)
    if events is not None:
        def sink(_instance_id, batches):
            c.ingest_kvbm_events([(kind, int(h)) for kind, hashes in batches for h in hashes])
            c.flush()
        events.add_sink(sink)
    return c
