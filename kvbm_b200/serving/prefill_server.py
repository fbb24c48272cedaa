"""A prefill instance served through the hub's prefill router.

``PrefillServer`` attaches a ``PrefillRouterHandler`` (registered on the hub
as a prefill worker, with its TTFT calibration) to a prefill
:class:`~kvbm_b200.serving.pd.PdInstance`: the hub's router calls the
handler's dispatch for a decode instance's remote prefill, the dispatch
puts the request on the instance's local plane, and the handler's
completion fires when the engine has finished the prefill (its KV is being
pushed into the decode pool; the decode side learns that it landed from its
mailbox). ``serve_forever`` steps the engine. Run it as

    python -m kvbm_b200.serving.prefill_server --hub http://HOST:PORT --instance-id N

for a Llama-architecture random-init model on the current GPU.

Parity: python/kvbm/vllm/prefill.py:35-45 (patches vLLM's build_and_serve to
attach the handler), src/hub/prefill_router.rs:132-245 (PrefillRouterHandler
with dispatch and calibrate lambdas), python/kvbm/hub/dispatch_lambda.py.
"""

from __future__ import annotations

import argparse
import threading

from ..engine.cd_plane import LocalPrefillPlane, decode_dispatch
from ..hub.client import CompletionEvent, PrefillRouterHandler


class PrefillServer:
    def __init__(self, instance, hub_url: str, max_concurrency: int = 8, calibrate=None, timeout: float = 300.0):
        if instance.role != "prefill":
            raise ValueError("PrefillServer serves a prefill instance")
        self.instance = instance
        self.local = instance.plane if isinstance(instance.plane, LocalPrefillPlane) else LocalPrefillPlane()
        instance.plane = self.local
        self._done: dict[str, CompletionEvent] = {}
        self._lock = threading.Lock()
        self.handler = PrefillRouterHandler(hub_url, self._dispatch, calibrate=calibrate,
                                            max_concurrency=max_concurrency, timeout=timeout)

    def _dispatch(self, request: dict, done: CompletionEvent) -> None:
        raw = bytes.fromhex(request["payload"])
        rid = decode_dispatch(raw)["request_id"]
        with self._lock:
            self._done[rid] = done
        self.local.dispatch(self.instance.instance_id, raw)

    def step(self) -> int:
        """Take routed requests, run one engine step; returns the prefills finished in it."""
        self.instance.pull()
        if not (self.instance.engine.has_unfinished() or self.instance.engine._delayed):
            return 0
        out = self.instance.step()
        for req in out:
            with self._lock:
                ev = self._done.pop(req.request_id, None)
            if ev is not None:
                ev.complete({"request_id": req.request_id, "prompt_tokens": req.num_prompt_tokens})
        return len(out)

    def serve_forever(self, stop: threading.Event | None = None, idle_wait_s: float = 0.005) -> None:
        stop = stop or threading.Event()
        while not stop.is_set():
            if not self.step():
                self.local.wait_nonempty(self.instance.instance_id, idle_wait_s)

    def close(self) -> None:
        self.handler.close()


def main(argv=None) -> None:
    import torch

    from ..engine.cd_plane import StorePeerDirectory
    from ..models.llama import LlamaConfig, LlamaModel
    from .pd import PdConfig, PdInstance

    p = argparse.ArgumentParser()
    p.add_argument("--hub", required=True)
    p.add_argument("--instance-id", type=int, required=True)
    p.add_argument("--store", default="127.0.0.1:29600", help="host:port of the deployment's key-value store")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--prompt-len", type=int, default=8192)
    a = p.parse_args(argv)
    import torch.distributed as dist

    host, port = a.store.rsplit(":", 1)
    store = dist.TCPStore(host, int(port), is_master=False)
    mcfg = LlamaConfig(layers=a.layers)
    model = LlamaModel(mcfg, torch.device("cuda", torch.cuda.current_device()))
    inst = PdInstance("prefill", model, PdConfig(model=mcfg, prompt_len=a.prompt_len), a.instance_id,
                      LocalPrefillPlane(), StorePeerDirectory(store), shared=True)
    server = PrefillServer(inst, a.hub)
    try:
        server.serve_forever()
    finally:
        server.close()
        inst.shutdown()


if __name__ == "__main__":
    main()
