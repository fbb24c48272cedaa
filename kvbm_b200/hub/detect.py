"""Attach a live vLLM engine to the hub's prefill router.

``try_wrap_engine(vllm_config, engine)`` looks at the engine's connector
configuration (``kv_transfer_config.kv_connector_extra_config``: the
block-manager configuration, with its ``default`` / ``leader`` profiles
applied) and, when it names a hub and the ``prefill`` disaggregation role,
registers the process as a prefill target: it returns a
:class:`PrefillRouterHandler` (with a calibrate handler when the engine's
limits can be read) whose dispatch lambda turns every routed
request into an ``engine.generate`` call (the prompt's token ids, one output
token, ``kv_transfer_params`` naming the decode instance that waits for the
KV) on the engine's event loop, and completes the router's call when that
generation ends. Without a hub, a prefill-role engine with a disaggregation
instance id is served from the node's prefill plane instead
(:class:`PlaneServer`). Decode or aggregated engines get ``None``.

Parity: python/kvbm/hub/detect.py (try_wrap_engine), the dispatch lambda of
python/kvbm/hub/dispatch_lambda.py, src/hub/prefill_router.rs:133-245.
"""

from __future__ import annotations

import asyncio
import logging
from typing import Any

from ..connector.leader import REMOTE_DECODE_KEY
from ..engine.cd_plane import decode_dispatch
from .client import CompletionEvent, PrefillRouterHandler

log = logging.getLogger(__name__)


def connector_settings(vllm_config: Any) -> tuple[str | None, str | None]:
    """(hub url, disaggregation role) from the engine's connector configuration."""
    ktc = getattr(vllm_config, "kv_transfer_config", None)
    extra = dict(getattr(ktc, "kv_connector_extra_config", None) or {})
    merged: dict = {}
    for layer in ({k: v for k, v in extra.items() if k not in ("default", "leader", "worker")},
                  extra.get("default") or {}, extra.get("leader") or {}):
        for k, v in layer.items():
            if isinstance(v, dict) and isinstance(merged.get(k), dict):
                merged[k] = {**merged[k], **v}
            else:
                merged[k] = v
    return (merged.get("hub") or {}).get("url"), (merged.get("disagg") or {}).get("role")


def _vllm_params(max_tokens: int, kv_transfer_params: dict):
    from vllm import SamplingParams

    return SamplingParams(max_tokens=max_tokens, extra_args={"kv_transfer_params": kv_transfer_params})


def make_dispatch_lambda(engine: Any, loop: asyncio.AbstractEventLoop, max_tokens: int = 1, make_params=None):
    """A dispatch lambda for :class:`PrefillRouterHandler`: runs each routed prefill as
    ``engine.generate`` on ``loop`` and completes the router's event when it finishes.
    ``make_params(max_tokens, kv_transfer_params)`` builds the sampling parameters (vLLM's by
    default)."""
    make_params = make_params or _vllm_params

    def dispatch(request: dict, done: CompletionEvent) -> None:
        d = decode_dispatch(bytes.fromhex(request["payload"]))
        params = dict(d["params"])
        params[REMOTE_DECODE_KEY] = d["decode"]

        async def run():
            sp = make_params(max_tokens, params)
            prompt = {"prompt_token_ids": [int(t) for t in d["tokens"]]}
            last = None
            async for out in engine.generate(prompt, sp, d["request_id"]):
                last = out
            return {"request_id": d["request_id"], "finished": bool(getattr(last, "finished", True))}

        fut = asyncio.run_coroutine_threadsafe(run(), loop)

        def finish(f):
            if f.exception() is not None:
                done.fail(f"{type(f.exception()).__name__}: {f.exception()}")
            else:
                done.complete(f.result())

        fut.add_done_callback(finish)

    return dispatch


class PlaneServer:
    """Serves a prefill engine from the node's prefill plane when there is no hub: a thread takes
    the dispatches addressed to ``instance_id`` (up to ``max_concurrency`` in flight) and hands each
    to ``dispatch`` (the same lambda the hub's router would call)."""

    def __init__(self, plane, instance_id: int, dispatch, max_concurrency: int = 4, poll_s: float = 0.2):
        import threading

        from ..engine.cd_plane import encode_dispatch

        self.plane, self.instance_id, self.dispatch = plane, int(instance_id), dispatch
        self.max_concurrency, self.poll_s = max_concurrency, poll_s
        self._encode = encode_dispatch
        self._inflight: list[CompletionEvent] = []
        self.served = 0
        self.failed = 0
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True, name="kvbm-plane-server")
        self._t.start()

    def _run(self) -> None:
        while not self._stop.is_set():
            done = [e for e in self._inflight if e.is_set()]
            self.failed += sum(1 for e in done if e.error is not None)
            self._inflight = [e for e in self._inflight if not e.is_set()]
            room = self.max_concurrency - len(self._inflight)
            if room <= 0:
                self._stop.wait(0.002)
                continue
            for d in self.plane.wait(self.instance_id, self.poll_s, limit=room):
                raw = self._encode(d["request_id"], d["tokens"], d["params"], d["decode"], salt=d.get("salt"),
                                   lora=d.get("lora"))
                ev = CompletionEvent()
                self._inflight.append(ev)
                self.served += 1
                try:
                    self.dispatch({"payload": raw.hex()}, ev)
                except Exception as e:  # noqa: BLE001 - one bad dispatch does not stop the server
                    ev.fail(f"{type(e).__name__}: {e}")

    def close(self) -> None:
        self._stop.set()
        self._t.join(timeout=2)


def try_wrap_engine(vllm_config: Any, engine: Any, loop: asyncio.AbstractEventLoop | None = None,
                    max_concurrency: int = 4, make_params=None) -> PrefillRouterHandler | PlaneServer | None:
    hub_url, role = connector_settings(vllm_config)
    if role != "prefill":
        return None
    if not hub_url:
        # no hub: serve the node's prefill plane under this engine's disaggregation instance id
        from ..engine.cd_plane import open_cd_services
        from ..utils.config import KvbmConfig

        ktc = getattr(vllm_config, "kv_transfer_config", None)
        cfg = KvbmConfig.for_leader(dict(getattr(ktc, "kv_connector_extra_config", None) or {}), env={},
                                    system_toml=None)
        if cfg.disagg is None or cfg.disagg.instance_id is None:
            return None
        loop = loop or asyncio.get_running_loop()
        plane, _ = open_cd_services(cfg.disagg.directory)
        server = PlaneServer(plane, cfg.disagg.instance_id, make_dispatch_lambda(engine, loop, make_params=make_params),
                             max_concurrency=max_concurrency)
        log.info("prefill plane attached (instance %s, %s)", cfg.disagg.instance_id, cfg.disagg.directory)
        return server
    loop = loop or asyncio.get_running_loop()
    # the calibrate handler is best effort: an engine whose limits cannot be read still serves prefills
    cal_lambda = cal_defaults = None
    try:
        from .calibrate_lambda import capture_calibration_defaults, make_calibrate_lambda

        mc = getattr(vllm_config, "model_config", None)
        model_id = str(getattr(mc, "served_model_name", None) or getattr(mc, "model", "") or "")
        cal_defaults = capture_calibration_defaults(engine, model_id)
        cal_lambda = make_calibrate_lambda(engine, loop)
    except Exception as e:  # noqa: BLE001
        log.info("prefill router: no calibrate handler (%s: %s)", type(e).__name__, e)
    handler = PrefillRouterHandler(hub_url, make_dispatch_lambda(engine, loop, make_params=make_params),
                                   max_concurrency=max_concurrency, calibrate_lambda=cal_lambda,
                                   calibration_defaults=cal_defaults)
    log.info("prefill router attached (instance %s, hub %s)", handler.instance_id, hub_url)
    return handler
