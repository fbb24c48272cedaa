"""The hub: one coordination service per deployment (HTTP/JSON, aiohttp).

Features (all in one process):

* discovery / registry - register, heartbeat (TTL eviction), deregister,
  peer lookup by instance or worker id;
* indexer - ingests KV-event batches from connector leaders into the native
  position-bucketed index and answers "which instance holds the deepest
  prefix of these hashes";
* disagg - the conditional-disaggregation prefill queue;
* prefill router - load-aware selection of prefill workers, circuit breaker,
  TTFT/ITL calibration, and dispatch of remote-prefill requests to a prefill
  worker's handler over the messenger;
* control / metrics - per-instance describe, metrics snapshot fan-in, a
  small status page.

Parity: crates/kvbm-hub/src/{server.rs (discovery port 1337, control 8337),
registry.rs, handlers.rs, features/indexer/*, features/disagg/*,
features/prefill_router/*, features/control_plane/manager.rs, web.rs}.
"""

from __future__ import annotations

import asyncio
import collections
import json
import os
import threading
import time

from aiohttp import web

from .. import _core_native as core
from ..runtime.messenger import Messenger
from .calibration import CALIBRATE_HANDLER, samples_from_traces
from .prefill_router import BreakerTicker, Calibration, CircuitBreaker, Selector
from .registry import InstanceRecord, InstanceRegistry

DEFAULT_DISCOVERY_PORT = 1337
DEFAULT_CONTROL_PORT = 8337
DISPATCH_HANDLER = "kvbm.prefill_router.dispatch"

WEB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "web")
WEB_ASSETS = {"/": ("index.html", "text/html"), "/app.js": ("app.js", "application/javascript"),
              "/style.css": ("style.css", "text/css")}


def _h(x) -> int:
    return int(x) if not isinstance(x, str) else int(x, 0)


class HubServer:
    def __init__(self, host: str = "127.0.0.1", port: int = 0, block_size: int = 16, max_seq_len: int = 0,
                 ttl: float = 30.0, features=("indexer", "p2p", "disagg", "prefill_router"),
                 max_inflight_per_worker: int = 4, breaker: bool = True, control_port: int | None = None,
                 messenger_port: int | None = None, layout: str = "operational",
                 advertise_host: str | None = None, g2_memory_gb: float = 0.0):
        self.host, self.port = host, port
        # the control port serves health, metrics and the status page apart from
        # the discovery / data routes (None: everything on the discovery port)
        self.control_port = control_port
        self.messenger_port = messenger_port
        self.layout, self.advertise_host, self.g2_memory_gb = layout, advertise_host or host, g2_memory_gb
        self.block_size, self.max_seq_len = block_size, max_seq_len
        self.features = list(features)
        self.index = core.PositionalIndex(max_seq_len - max_seq_len % block_size, block_size)
        self.registry = InstanceRegistry(ttl=ttl, on_evict=self._on_evict)
        self.selector = Selector(max_inflight_per_worker, block_size)
        self.breaker = CircuitBreaker() if breaker else None
        self._ticker = None
        self.calibration: dict[int, Calibration] = collections.defaultdict(Calibration)
        self.cd_queue: collections.deque = collections.deque()
        self.counters = collections.Counter()
        self.messenger: Messenger | None = None
        self._loop = None
        self._runner = None
        self._thread = None
        self._started = threading.Event()

    # ------------------------------------------------------------ wiring
    def _on_evict(self, instance_id: int) -> None:
        self.index.remove_instance(instance_id)
        self.selector.remove_worker(instance_id)
        self.counters["evictions"] += 1

    def app(self) -> web.Application:
        a = web.Application()
        r = a.router
        for path in WEB_ASSETS:
            r.add_get(path, self._asset)
        r.add_get("/health", self._health)
        r.add_get("/v1/config", self._config)
        r.add_post("/v1/instances", self._register)
        r.add_get("/v1/instances", self._list)
        r.add_delete("/v1/instances/{iid}", self._unregister)
        r.add_post("/v1/instances/{iid}/heartbeat", self._heartbeat)
        r.add_get("/v1/instances/{iid}/describe", self._describe)
        r.add_get("/v1/peers/instance/{iid}", self._peer_instance)
        r.add_get("/v1/peers/worker/{wid}", self._peer_worker)
        r.add_post("/v1/indexer/events", self._events)
        r.add_post("/v1/indexer/query", self._query)
        r.add_get("/v1/indexer/config", self._index_config)
        r.add_get("/v1/indexer/instances", self._index_instances)
        r.add_get("/v1/indexer/hashes/by_position", self._index_by_position)
        r.add_post("/v1/disagg/enqueue", self._cd_enqueue)
        r.add_post("/v1/disagg/dequeue", self._cd_dequeue)
        r.add_get("/v1/disagg/instances", self._cd_instances)
        r.add_get("/v1/prefill-router/targets", self._targets)
        r.add_get("/v1/prefill-router/counters", self._router_counters)
        r.add_post("/v1/prefill-router/calibrate/{iid}", self._calibrate)
        r.add_post("/v1/prefill-router/dispatch", self._dispatch)
        r.add_get("/v1/metrics", self._metrics)
        return a

    # ----------------------------------------------------------- handlers
    async def _health(self, req):
        return web.json_response({"status": "ok", "time": time.time()})

    async def _targets(self, req):
        return web.json_response({"targets": self.selector.targets()})

    async def _asset(self, req):
        name, ctype = WEB_ASSETS[req.path]
        with open(os.path.join(WEB_DIR, name), encoding="utf-8") as f:
            return web.Response(text=f.read(), content_type=ctype)

    async def _config(self, req):
        return web.json_response({"block_size": self.block_size, "max_seq_len": self.max_seq_len,
                                  "features": self.features, "ttl": self.registry.ttl, "layout": self.layout,
                                  "advertise_host": self.advertise_host, "g2_memory_gb": self.g2_memory_gb,
                                  "control_port": self.control_port,
                                  "messenger": self.messenger.address if self.messenger else None})

    def control_app(self) -> web.Application:
        a = web.Application()
        for path in WEB_ASSETS:
            a.router.add_get(path, self._asset)
        a.router.add_get("/health", self._health)
        a.router.add_get("/v1/config", self._config)
        a.router.add_get("/v1/metrics", self._metrics)
        a.router.add_get("/v1/instances", self._list)
        return a

    async def _register(self, req):
        d = await req.json()
        if d.get("block_size", self.block_size) != self.block_size:
            return web.json_response({"error": "block_size mismatch", "hub_block_size": self.block_size},
                                     status=409)
        rec = InstanceRecord(instance_id=_h(d["instance_id"]), address=d.get("address", ""),
                             role=d.get("role", "both"), features=d.get("features", []),
                             workers=d.get("workers", {}), block_size=self.block_size,
                             max_seq_len=d.get("max_seq_len"), layout=d.get("layout", {}))
        self.registry.register(rec)
        if rec.max_seq_len:
            self.index.grow_to_max_seq_len(rec.max_seq_len - rec.max_seq_len % self.block_size)
        if rec.role in ("prefill", "both") and "prefill_router" in rec.features:
            self.selector.add_worker(rec.instance_id, d.get("max_inflight"))
        self.counters["registrations"] += 1
        return web.json_response({"ok": True, "ttl": self.registry.ttl, "hub": self.features})

    async def _list(self, req):
        role = req.query.get("role")
        return web.json_response({"instances": [r.public() for r in self.registry.list(role=role)]})

    async def _unregister(self, req):
        return web.json_response({"ok": self.registry.unregister(_h(req.match_info["iid"]))})

    async def _heartbeat(self, req):
        ok = self.registry.heartbeat(_h(req.match_info["iid"]))
        return web.json_response({"ok": ok}, status=200 if ok else 404)

    async def _describe(self, req):
        rec = self.registry.get(_h(req.match_info["iid"]))
        if rec is None:
            return web.json_response({"error": "unknown instance"}, status=404)
        return web.json_response(rec.public())

    async def _peer_instance(self, req):
        rec = self.registry.get(_h(req.match_info["iid"]))
        if rec is None:
            return web.json_response({"error": "unknown instance"}, status=404)
        return web.json_response({"instance_id": str(rec.instance_id), "address": rec.address,
                                  "workers": rec.workers})

    async def _peer_worker(self, req):
        got = self.registry.peer_by_worker(req.match_info["wid"])
        if got is None:
            return web.json_response({"error": "unknown worker"}, status=404)
        return web.json_response({"instance_id": str(got[0]), "address": got[1]})

    async def _events(self, req):
        d = await req.json()
        iid = _h(d["instance_id"])
        if self.registry.get(iid) is None:
            return web.json_response({"error": "unregistered instance"}, status=404)
        for kind, hashes in d["batches"]:
            self.index.apply(iid, kind, [_h(h) for h in hashes])
            self.counters[f"events_{kind}"] += len(hashes)
        return web.json_response({"ok": True})

    async def _query(self, req):
        d = await req.json()
        got = self.index.query_holders([_h(h) for h in d["hashes"]])
        self.counters["queries"] += 1
        if got is None:
            return web.json_response({"hit": False})
        h, holders = got
        return web.json_response({"hit": True, "hash": str(h), "position": h >> 128,
                                  "holders": [str(x) for x in holders]})

    async def _index_config(self, req):
        return web.json_response({"block_size": self.block_size, "num_positions": self.index.num_positions(),
                                  "dropped_out_of_range": self.index.dropped_out_of_range(),
                                  "entries": self.index.num_entries()})

    async def _index_by_position(self, req):
        """Every indexed block at one position bucket: its lineage word, the sequence hash that a
        query names (position, lineage; the index does not keep the parent word) and its holders."""
        try:
            pos = int(req.query["position"])
        except (KeyError, ValueError):
            return web.json_response({"error": "position=<int> is required"}, status=400)
        rows = self.index.by_position(pos)
        return web.json_response({"position": pos, "blocks": [
            {"lineage": str(lin), "hash_u128": str((pos << 128) | lin), "holders": [str(h) for h in holders]}
            for lin, holders in rows]})

    async def _index_instances(self, req):
        return web.json_response({"instances": [str(r.instance_id) for r in self.registry.list(feature="indexer")]})

    async def _cd_enqueue(self, req):
        d = await req.json()
        self.cd_queue.append(d)
        self.counters["cd_enqueued"] += 1
        return web.json_response({"ok": True, "depth": len(self.cd_queue)})

    async def _cd_dequeue(self, req):
        if not self.cd_queue:
            return web.json_response({"request": None})
        self.counters["cd_dequeued"] += 1
        return web.json_response({"request": self.cd_queue.popleft()})

    async def _cd_instances(self, req):
        return web.json_response({"prefill": [str(r.instance_id) for r in self.registry.list(role="prefill")],
                                  "decode": [str(r.instance_id) for r in self.registry.list(role="decode")],
                                  "queue_depth": len(self.cd_queue)})

    async def _router_counters(self, req):
        return web.json_response({"counters": dict(self.counters),
                                  "breaker": int(self.breaker.tier) if self.breaker else None,
                                  "pressure": self.selector.pressure(),
                                  "calibration": {str(k): v.to_dict() for k, v in self.calibration.items()}})

    async def _calibrate(self, req):
        """Either measured samples (``ttft`` / ``itl`` lists) for an instance's models, or a
        calibration request proxied to that prefill worker (``request``, ``?force=true``): the
        worker runs its sweep and the fitted traces feed the instance's models here too.
        409 when the worker is busy with prefills or another sweep."""
        d = await req.json()
        iid = _h(req.match_info["iid"])
        cal = self.calibration[iid]
        if "ttft" in d or "itl" in d:
            for isl, s in d.get("ttft", []):
                cal.add_ttft(isl, s)
            for ctx, s in d.get("itl", []):
                cal.add_itl(ctx, s)
            return web.json_response(cal.to_dict())
        rec = self.registry.get(iid)
        if rec is None:
            return web.json_response({"error": f"unknown instance {iid}"}, status=404)
        if self.messenger is None:
            return web.json_response({"error": "this hub has no messenger to reach workers"}, status=503)
        force = req.query.get("force", "false").lower() in ("1", "true", "yes")
        timeout = float(d.get("timeout", 1800.0))
        loop = asyncio.get_running_loop()
        try:
            out = await loop.run_in_executor(None, lambda: self.messenger.call(
                rec.address, CALIBRATE_HANDLER, {"request": d.get("request") or {}, "force": force}, timeout=timeout))
        except Exception as e:  # noqa: BLE001 - the worker's refusal or failure goes back to the caller
            msg = str(e)
            busy = "already_calibrating" in msg or "prefill_busy" in msg
            return web.json_response({"error": msg}, status=409 if busy else 502)
        if not out.get("from_cache"):
            ttft, itl = samples_from_traces(out["results"]["traces"])
            for isl, s in ttft:
                cal.add_ttft(isl, s)
            for ctx, s in itl:
                cal.add_itl(ctx, s)
        self.counters["calibrations"] += 1
        return web.json_response(out)

    async def _dispatch(self, req):
        d = await req.json()
        loop = asyncio.get_running_loop()
        try:
            res = await loop.run_in_executor(None, self.dispatch_blocking, d)
        except TimeoutError as e:
            return web.json_response({"error": str(e)}, status=503)
        return web.json_response(res)

    def dispatch_blocking(self, d: dict) -> dict:
        charge = self.selector.pick(int(d.get("num_tokens", 0)), int(d.get("num_provided_tokens", 0)),
                                    timeout=float(d.get("timeout", 30.0)))
        with charge:
            rec = self.registry.get(charge.slot.instance_id)
            self.counters["dispatched"] += 1
            if rec is None or self.messenger is None:
                return {"instance_id": str(charge.slot.instance_id), "forwarded": False}
            out = self.messenger.call(rec.address, DISPATCH_HANDLER, d.get("request", {}),
                                      timeout=float(d.get("timeout", 30.0)))
            return {"instance_id": str(charge.slot.instance_id), "forwarded": True, "result": out}

    async def _metrics(self, req):
        return web.json_response({"instances": len(self.registry.list()), "counters": dict(self.counters),
                                  "index_entries": self.index.num_entries()})

    # ------------------------------------------------------------ running
    async def _sweeper(self):
        while True:
            await asyncio.sleep(max(0.02, self.registry.ttl / 4))
            self.registry.sweep()

    def _serve(self):
        self._loop = asyncio.new_event_loop()
        asyncio.set_event_loop(self._loop)

        async def start():
            self._runner = web.AppRunner(self.app())
            await self._runner.setup()
            site = web.TCPSite(self._runner, self.host, self.port)
            await site.start()
            self.port = site._server.sockets[0].getsockname()[1]
            if self.control_port is not None:
                self._control_runner = web.AppRunner(self.control_app())
                await self._control_runner.setup()
                csite = web.TCPSite(self._control_runner, self.host, self.control_port)
                await csite.start()
                self.control_port = csite._server.sockets[0].getsockname()[1]
            self._sweep_task = self._loop.create_task(self._sweeper())
            self._started.set()

        self._loop.run_until_complete(start())
        self._loop.run_forever()

    def start(self) -> "HubServer":
        bind = f"tcp://{self.host}:{self.messenger_port}" if self.messenger_port is not None else "tcp://127.0.0.1:0"
        self.messenger = Messenger(bind=bind)
        if self.breaker is not None:
            self._ticker = BreakerTicker(self.breaker, self.selector)
        self._thread = threading.Thread(target=self._serve, daemon=True, name="kvbm-hub")
        self._thread.start()
        if not self._started.wait(10):
            raise RuntimeError("hub did not start")
        return self

    @property
    def url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def stop(self) -> None:
        if self._ticker:
            self._ticker.stop()
        if self._loop is not None:
            async def shutdown():
                task = getattr(self, "_sweep_task", None)
                if task is not None:
                    task.cancel()
                    try:
                        await task
                    except asyncio.CancelledError:
                        pass
                await self._runner.cleanup()
                if getattr(self, "_control_runner", None) is not None:
                    await self._control_runner.cleanup()
            fut = asyncio.run_coroutine_threadsafe(shutdown(), self._loop)
            try:
                fut.result(5)
            finally:
                self._loop.call_soon_threadsafe(self._loop.stop)
                self._thread.join(timeout=5)
        if self.messenger:
            self.messenger.close()


def main(argv=None) -> None:
    """``python -m kvbm_b200.hub.server`` (the ``kvbm_hub`` binary)."""
    import argparse

    p = argparse.ArgumentParser(description="kvbm hub")
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--discovery-port", type=int, default=DEFAULT_DISCOVERY_PORT)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--max-seq-len", type=int, default=131072)
    p.add_argument("--ttl", type=float, default=30.0)
    p.add_argument("--features", default="indexer,p2p,disagg,prefill_router")
    p.add_argument("--control-port", type=int, default=DEFAULT_CONTROL_PORT)
    p.add_argument("--velo-port", "--messenger-port", dest="messenger_port", type=int, default=None,
                   help="port of the hub's RPC messenger (prefill-router dispatch)")
    p.add_argument("--layout", default="operational", choices=["operational", "universal"])
    p.add_argument("--kv-index-advertise-host", default=None)
    p.add_argument("--g2-memory", type=float, default=0.0, help="GB of host memory the hub reports for P2P staging")
    a = p.parse_args(argv)
    hub = HubServer(a.host, a.discovery_port, a.block_size, a.max_seq_len, a.ttl, a.features.split(","),
                    control_port=a.control_port, messenger_port=a.messenger_port, layout=a.layout,
                    advertise_host=a.kv_index_advertise_host, g2_memory_gb=a.g2_memory).start()
    print(json.dumps({"hub": hub.url, "control": f"http://{a.host}:{hub.control_port}"}), flush=True)
    try:
        while True:
            time.sleep(3600)
    except KeyboardInterrupt:
        hub.stop()


if __name__ == "__main__":
    main()
