"""Hub client, registration guard and the prefill-worker side of routing.

* :class:`HubClient` - JSON/HTTP calls to the hub (register, heartbeat,
  events, indexer query, CD queue, router dispatch/calibration).
* :class:`HubRegistration` - registers an instance, heartbeats on a
  background thread, and deregisters (HTTP DELETE) when closed or garbage
  collected (the reference's RAII HubRegistrationGuard).
* :class:`PrefillRouterHandler` / :class:`CompletionEvent` - run in a prefill
  worker process: own a messenger participant, serve the hub's dispatch
  calls by invoking a user ``dispatch`` lambda, and signal completion.

Parity: crates/kvbm-hub/src/client.rs (HubClient + DELETE guard),
src/hub/prefill_router.rs:63-245 (CompletionEvent, PrefillRouterHandler),
python/kvbm/hub/{dispatch_lambda,calibrate_lambda,detect}.py.
"""

from __future__ import annotations

import threading
import time
import uuid
import weakref
from typing import Any, Callable

import requests

from ..runtime.messenger import Messenger
from .server import DISPATCH_HANDLER


class HubClient:
    def __init__(self, url: str, timeout: float = 10.0):
        self.url = url.rstrip("/")
        self.timeout = timeout
        self.s = requests.Session()

    def _req(self, method: str, path: str, **kw):
        r = self.s.request(method, self.url + path, timeout=kw.pop("timeout", self.timeout), **kw)
        if r.status_code >= 400:
            raise RuntimeError(f"hub {method} {path}: {r.status_code} {r.text}")
        return r.json()

    def health(self) -> dict:
        return self._req("GET", "/health")

    def config(self) -> dict:
        return self._req("GET", "/v1/config")

    def register(self, instance_id: int, **info) -> dict:
        return self._req("POST", "/v1/instances", json={"instance_id": str(instance_id), **info})

    def heartbeat(self, instance_id: int) -> bool:
        try:
            return bool(self._req("POST", f"/v1/instances/{instance_id}/heartbeat").get("ok"))
        except RuntimeError:
            return False

    def unregister(self, instance_id: int) -> bool:
        return bool(self._req("DELETE", f"/v1/instances/{instance_id}").get("ok"))

    def instances(self, role: str | None = None) -> list[dict]:
        return self._req("GET", "/v1/instances", params={"role": role} if role else None)["instances"]

    def peer(self, instance_id: int) -> dict:
        return self._req("GET", f"/v1/peers/instance/{instance_id}")

    def publish_events(self, instance_id: int, batches: list[tuple[str, list[int]]]) -> None:
        self._req("POST", "/v1/indexer/events",
                  json={"instance_id": str(instance_id), "batches": [[k, [str(h) for h in hs]] for k, hs in batches]})

    def query(self, hashes: list[int]) -> dict:
        d = self._req("POST", "/v1/indexer/query", json={"hashes": [str(h) for h in hashes]})
        if d.get("hit"):
            d["hash"] = int(d["hash"])
            d["holders"] = [int(x) for x in d["holders"]]
        return d

    def cd_enqueue(self, request: dict) -> dict:
        return self._req("POST", "/v1/disagg/enqueue", json=request)

    def cd_dequeue(self) -> dict | None:
        return self._req("POST", "/v1/disagg/dequeue", json={})["request"]

    def dispatch(self, num_tokens: int, num_provided_tokens: int, request: dict, timeout: float = 30.0) -> dict:
        return self._req("POST", "/v1/prefill-router/dispatch",
                         json={"num_tokens": num_tokens, "num_provided_tokens": num_provided_tokens,
                               "request": request, "timeout": timeout}, timeout=timeout + 5)

    def calibrate(self, instance_id: int, ttft=(), itl=()) -> dict:
        """Post measured (tokens, seconds) samples for a prefill instance's TTFT / ITL models."""
        return self._req("POST", f"/v1/prefill-router/calibrate/{instance_id}",
                         json={"ttft": list(ttft), "itl": list(itl)})

    def run_calibration(self, instance_id: int, request: dict | None = None, force: bool = False,
                        timeout: float = 1800.0) -> dict:
        """Ask a prefill worker to run a calibration sweep (``CalibrationRequest`` fields, all
        optional); returns the fitted model, the resolved knobs and whether it was cached."""
        return self._req("POST", f"/v1/prefill-router/calibrate/{instance_id}",
                         params={"force": "true" if force else "false"},
                         json={"request": request or {}, "timeout": timeout}, timeout=timeout + 10)

    def index_config(self) -> dict:
        return self._req("GET", "/v1/indexer/config")

    def index_instances(self) -> list[str]:
        return self._req("GET", "/v1/indexer/instances")["instances"]

    def index_by_position(self, position: int) -> dict:
        return self._req("GET", "/v1/indexer/hashes/by_position", params={"position": int(position)})

    def disagg_instances(self) -> dict:
        return self._req("GET", "/v1/disagg/instances")

    def router_counters(self) -> dict:
        return self._req("GET", "/v1/prefill-router/counters")

    def targets(self) -> list[dict]:
        return self._req("GET", "/v1/prefill-router/targets")["targets"]


class HubRegistration:
    """Register + heartbeat; deregisters on close() or garbage collection."""

    def __init__(self, client: HubClient, instance_id: int, heartbeat_s: float = 5.0, **info):
        self.client, self.instance_id = client, instance_id
        client.register(instance_id, **info)
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._beat, args=(heartbeat_s,), daemon=True, name="kvbm-hub-hb")
        self._t.start()
        self._fin = weakref.finalize(self, _deregister, client, instance_id, self._stop)

    def _beat(self, period):
        while not self._stop.wait(period):
            if not self.client.heartbeat(self.instance_id):
                pass  # the hub forgot us (TTL): the next register() call restores it

    def close(self) -> None:
        self._fin()
        self._t.join(timeout=2)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _deregister(client: HubClient, instance_id: int, stop: threading.Event) -> None:
    stop.set()
    try:
        client.unregister(instance_id)
    except Exception:  # noqa: BLE001 - best effort at shutdown
        pass


class CompletionEvent:
    """A one-shot completion a dispatch lambda signals when its prefill is done."""

    def __init__(self):
        self._ev = threading.Event()
        self.result: Any = None
        self.error: str | None = None

    def complete(self, result: Any = None) -> None:
        self.result = result
        self._ev.set()

    def fail(self, error: str) -> None:
        self.error = error
        self._ev.set()

    def wait(self, timeout: float | None = None) -> Any:
        if not self._ev.wait(timeout):
            raise TimeoutError("prefill did not complete in time")
        if self.error is not None:
            raise RuntimeError(self.error)
        return self.result

    def is_set(self) -> bool:
        return self._ev.is_set()


class PrefillRouterHandler:
    """Prefill-worker side: serves the hub's dispatch calls.

    ``dispatch(request: dict, done: CompletionEvent)`` starts the prefill
    (e.g. by calling the engine's generate with the request's
    kv_transfer_params) and completes ``done`` when the KV is available to
    the decode side. Only one dispatch runs at a time per handler unless
    ``max_concurrency`` says otherwise (mutual exclusion counters).
    """

    def __init__(self, hub_url: str, dispatch: Callable[[dict, CompletionEvent], None],
                 calibrate: Callable[[], dict] | None = None, instance_id: int | None = None,
                 max_concurrency: int = 4, timeout: float = 60.0,
                 calibrate_lambda: Callable[[dict, CompletionEvent], None] | None = None,
                 calibration_defaults: dict | None = None, calibration_timeout: float = 1800.0):
        from .calibration import CALIBRATE_HANDLER, CalibrationDefaults

        self.instance_id = instance_id if instance_id is not None else uuid.uuid4().int >> 64
        self.messenger = Messenger(self.instance_id)
        self.dispatch_fn, self.calibrate_fn = dispatch, calibrate
        self.timeout = timeout
        self.max_concurrency = max_concurrency
        self.inflight = 0
        self.completed = 0
        self._lock = threading.Lock()
        # hub-triggered calibration sweeps: never while a prefill runs, no prefill while one runs
        self.calibrate_lambda = calibrate_lambda
        self.calibration_defaults = CalibrationDefaults.from_dict(calibration_defaults)
        self.calibration_timeout = calibration_timeout
        self.calibrating = False
        self._calibration: dict | None = None  # the last analysed sweep (returned again unless forced)
        self.messenger.register_handler(DISPATCH_HANDLER, self._on_dispatch)
        if calibrate_lambda is not None:
            self.messenger.register_handler(CALIBRATE_HANDLER, self._on_calibrate)
        self.client = HubClient(hub_url)
        self.registration = HubRegistration(self.client, self.instance_id, role="prefill",
                                            features=["prefill_router"], address=self.messenger.address,
                                            max_inflight=max_concurrency)
        if calibrate is not None:
            cal = calibrate()
            self.client.calibrate(self.instance_id, cal.get("ttft", ()), cal.get("itl", ()))

    def _on_calibrate(self, payload: dict | None):
        """Run (or return the cached) calibration sweep: resolve the caller's knobs against the
        engine's limits, hand them to the calibrate lambda, fit the traces it returns."""
        from .calibration import CalibrationRequest, analyze

        req = CalibrationRequest.from_dict((payload or {}).get("request"))
        force = bool((payload or {}).get("force")) or req.force
        with self._lock:
            if self._calibration is not None and not force:
                return {**self._calibration, "from_cache": True}
            if self.calibrating:
                raise RuntimeError("already_calibrating")
            if self.inflight:
                raise RuntimeError(f"prefill_busy ({self.inflight} in flight)")
            self.calibrating = True
        try:
            resolved = req.resolve(self.calibration_defaults)
            done = CompletionEvent()
            self.calibrate_lambda(resolved.to_dict(), done)
            raw = done.wait(self.calibration_timeout)
            out = {"results": analyze(list(raw["traces"])), "resolved": resolved.to_dict(),
                   "defaults": dict(vars(self.calibration_defaults))}
            with self._lock:
                self._calibration = out
            return {**out, "from_cache": False}
        finally:
            with self._lock:
                self.calibrating = False

    def _on_dispatch(self, request: dict):
        with self._lock:
            if self.calibrating:
                raise RuntimeError("calibration_in_progress")
            if self.inflight >= self.max_concurrency:
                raise RuntimeError("prefill handler saturated")
            self.inflight += 1
        done = CompletionEvent()
        t0 = time.monotonic()
        try:
            self.dispatch_fn(request, done)
            result = done.wait(self.timeout)
        finally:
            with self._lock:
                self.inflight -= 1
                self.completed += 1
        return {"result": result, "seconds": time.monotonic() - t0}

    def close(self) -> None:
        self.registration.close()
        self.messenger.close()
