"""The binding surface the reference exposes as ``kvbm._core``.

Classes: ``KvbmRuntime`` (config + messenger + optional hub registration;
``build_leader`` / ``build_worker``), ``ConnectorLeader``,
``ConnectorWorker``, ``KvbmRequest``, ``SchedulerOutput`` (builder),
``Tensor`` (data_ptr/shape/stride/device view), ``KvbmVllmConfig``;
functions ``is_available``; submodule ``hub`` with ``PrefillRouterHandler``
and ``CompletionEvent``.

Parity: src/lib.rs:74-105 (module contents), src/runtime.rs:57-177
(build_worker, build_leader, peer_info, register_peer),
src/connector/leader/mod.rs:40-347, leader/request.rs:8,
leader/scheduler.rs:18-122, src/connector/worker/mod.rs:26-342,
src/torch/mod.rs:140, src/vllm/config.rs:246, src/hub/prefill_router.rs.
"""

from __future__ import annotations

import time
import types

from . import __version__
from .connector.leader import ConnectorLeader as _Leader
from .connector.leader import KvbmRequest
from .connector.leader import SchedulerOutputLite
from .engine.leader import InstanceLeader, ParallelWorkers
from .hub import client as _hub_client
from .logical.manager import BlockManager, Tier
from .runtime.messenger import Messenger
from .utils.config import KvbmConfig

LAYOUT_HANDLER = "kvbm.connector.worker.get_layout_config"
HANDLERS_HANDLER = "kvbm.runtime.handlers"   # the handler names a runtime's messenger serves


def is_available() -> bool:
    """True when the native core and the CUDA kernel library load."""
    try:
        from . import _core_native  # noqa: F401
        from .ops import _lib

        _lib.load(build_if_missing=False)
        return True
    except Exception:  # noqa: BLE001
        return False


class KvbmRuntime:
    def __init__(self, config: KvbmConfig, role: str):
        self.config, self.role = config, role
        self.messenger = Messenger(bind=config.messenger.bind)
        self.messenger.register_handler(HANDLERS_HANDLER, lambda _p: sorted(self.messenger._handlers))
        for iid, addr in (config.messenger.peers or {}).items():  # static discovery
            self.messenger.register_peer(int(iid), addr)
        self.hub = None
        self._registration = None
        if config.hub is not None and config.hub.url:
            self.hub = _hub_client.HubClient(config.hub.url)

    def register_with_hub(self, features=("indexer", "p2p"), **info):
        """Register this instance on the hub and keep it alive with heartbeats (until shutdown)."""
        if self.hub is None:
            raise RuntimeError("no hub configured (hub.url)")
        self._registration = _hub_client.HubRegistration(
            self.hub, self.messenger.instance_id, heartbeat_s=self.config.hub.heartbeat_secs,
            features=list(features), address=self.messenger.address, role=self.role, **info)
        return self._registration

    @classmethod
    def build_leader(cls, json_config: str | None = None) -> "KvbmRuntime":
        return cls(KvbmConfig.for_leader(json_config), "leader")

    @classmethod
    def build_worker(cls, json_config: str | None = None) -> "KvbmRuntime":
        return cls(KvbmConfig.for_worker(json_config), "worker")

    def instance_id(self) -> bytes:
        return self.messenger.instance_id.to_bytes(16, "big")

    def peer_info(self) -> tuple[int, str]:
        return self.messenger.instance_id, self.messenger.address

    def register_peer(self, instance_id: int, address: str) -> None:
        self.messenger.register_peer(instance_id, address)

    def wait_for_handler(self, instance_id: int, handler_name: str, timeout_s: float = 60.0) -> None:
        """Block until peer ``instance_id`` serves ``handler_name`` (its messenger lists it)."""
        deadline = time.monotonic() + timeout_s
        last = None
        while time.monotonic() < deadline:
            try:
                if handler_name in self.messenger.call(int(instance_id), HANDLERS_HANDLER, None, timeout=2.0):
                    return
            except Exception as e:  # noqa: BLE001 - the peer may not be up yet
                last = e
            time.sleep(0.05)
        raise TimeoutError(f"peer {instance_id} did not serve {handler_name!r} within {timeout_s} s ({last})")

    def shutdown(self) -> None:
        if self._registration is not None:
            self._registration.close()
            self._registration = None
        self.messenger.close()


class Tensor:
    """A framework tensor as the block manager sees it."""

    def __init__(self, t):
        self._t = t

    def data_ptr(self) -> int:
        return self._t.data_ptr()

    @property
    def shape(self) -> list[int]:
        return list(self._t.shape)

    @property
    def stride(self) -> list[int]:
        return list(self._t.stride())

    @property
    def device(self) -> int:
        return self._t.device.index if self._t.is_cuda else -1

    @property
    def element_size(self) -> int:
        return self._t.element_size()

    def torch(self):
        return self._t


class KvbmVllmConfig:
    """The vLLM facts the block manager sizes itself from.

    Built either from one flat mapping (``info``, this library's connector
    form) or, as the reference's binding is, from a ``parallel`` and an
    ``attention`` section (world size, ranks, TP/PP/DP degrees; block size,
    block counts, cache dtype bytes, KV layout, head size, KV heads); both
    forms expose ``info`` (flat), ``parallel`` and ``attention``."""

    def __init__(self, info_or_parallel: dict | None = None, attention: dict | None = None):
        if attention is None:
            self.info = dict(info_or_parallel or {})
            self.parallel = {k: self.info[k] for k in ("world_size", "rank", "tensor_parallel_size",
                                                       "pipeline_parallel_size", "data_parallel_size",
                                                       "data_parallel_rank") if k in self.info}
            self.attention = {k: self.info[k] for k in ("block_size", "head_size", "num_kv_heads", "dtype_bytes",
                                                        "cache_dtype", "num_layers") if k in self.info}
        else:
            self.parallel, self.attention = dict(info_or_parallel or {}), dict(attention)
            self.info = {**self.parallel, **self.attention}

    def __eq__(self, other) -> bool:
        return isinstance(other, KvbmVllmConfig) and self.info == other.info

    def __repr__(self) -> str:
        return f"KvbmVllmConfig(parallel={self.parallel}, attention={self.attention})"

    @classmethod
    def from_vllm(cls, vllm_config) -> "KvbmVllmConfig":
        from .connector.config import extract_vllm_config_for_kvbm

        return cls(extract_vllm_config_for_kvbm(vllm_config))


class SchedulerOutput:
    """Builder for one scheduler step (what vLLM's SchedulerOutput carries)."""

    def __init__(self, iteration: int = 0):
        self.iteration = iteration
        self._lite = SchedulerOutputLite(step=iteration)
        self._sched: dict[str, int] = {}

    def add_new_request(self, request_id: str, prompt_token_ids: list[int], block_ids: list[int],
                        num_computed_tokens: int) -> None:
        self._lite.scheduled[request_id] = ([], list(block_ids), num_computed_tokens)

    def add_cached_request(self, request_id: str, new_token_ids: list[int], new_block_ids: list[int],
                           num_computed_tokens: int) -> None:
        self._lite.scheduled[request_id] = (list(new_token_ids), list(new_block_ids), num_computed_tokens)

    def add_num_scheduled_tokens(self, counts: dict[str, int]) -> None:
        self._sched.update(counts)

    def add_finished(self, request_ids: list[str]) -> None:
        self._lite.finished_req_ids.extend(request_ids)

    def set_num_scheduled_tokens(self, counts: dict[str, int]) -> None:
        self._sched = dict(counts)

    def get_total_num_scheduled_tokens(self) -> int:
        return sum(self._sched.values())

    def set_preempted_req_ids(self, request_ids) -> None:
        self._lite.preempted_req_ids = sorted(request_ids or [])

    def serialize(self) -> bytes:
        """The step as msgpack: iteration, per-request (new tokens, new blocks, computed tokens),
        scheduled token counts, finished and preempted ids."""
        import msgpack

        return msgpack.packb({"iteration": self.iteration,
                              "scheduled": {r: [list(t), list(b), int(c)] for r, (t, b, c) in
                                            self._lite.scheduled.items()},
                              "num_scheduled_tokens": dict(self._sched),
                              "finished": list(self._lite.finished_req_ids),
                              "preempted": list(self._lite.preempted_req_ids)}, use_bin_type=True)

    def lite(self) -> SchedulerOutputLite:
        out = SchedulerOutputLite(self.iteration)
        for rid, (toks, blocks, computed) in self._lite.scheduled.items():
            out.scheduled[rid] = (toks, blocks, computed + self._sched.get(rid, 0))
        out.finished_req_ids = list(self._lite.finished_req_ids)
        out.preempted_req_ids = list(self._lite.preempted_req_ids)
        return out


class ConnectorLeader:
    """Scheduler-side connector bound to a runtime; sized from the workers' layouts."""

    def __init__(self, runtime: KvbmRuntime, block_size: int, consolidator_endpoints=None):
        self.runtime, self.block_size = runtime, block_size
        self.consolidator_endpoints = consolidator_endpoints
        self._workers: dict[int, tuple[int, str]] = {}
        self._impl: _Leader | None = None

    def register_worker(self, rank: int, instance_id: int, address: str) -> None:
        self.runtime.register_peer(instance_id, address)
        self._workers[rank] = (instance_id, address)

    def initialize_workers(self, layout: dict | None = None) -> None:
        """Query one worker's layout (or use ``layout``) and build the G2/G3 pools."""
        if layout is None:
            if not self._workers:
                raise RuntimeError("no workers registered")
            iid, _ = self._workers[min(self._workers)]
            layout = self.runtime.messenger.call(iid, LAYOUT_HANDLER)
        cfg = self.runtime.config
        g2n = max(1, int(layout.get("g2_blocks", 0)))
        g3n = int(layout.get("g3_blocks", 0))
        g2 = BlockManager(g2n, self.block_size, cfg.cache.inactive_backend, Tier.G2,
                          duplicate_policy=cfg.cache.duplicate_policy)
        g3 = BlockManager(g3n, self.block_size, cfg.cache.inactive_backend, Tier.G3,
                          registry=g2.registry) if g3n else None
        # the registered workers (one per TP rank, each serving its shard) carry out the leader's own
        # block operations; per-step ops reach them through the connector metadata
        if self._workers:
            from .engine.spmd import SpmdParallelWorkers

            leader = InstanceLeader(g2, SpmdParallelWorkers(self.runtime.messenger,
                                                            [self._workers[r][0] for r in sorted(self._workers)]), g3=g3)
        else:
            leader = InstanceLeader.scheduler_side(g2, g3)
        objects = None
        if cfg.object is not None:
            from .object import make_object_store

            objects = make_object_store(cfg.object)
        from .connector.vllm_connector import disagg_leader_kwargs

        self._impl = _Leader(leader, self.block_size, objects=objects,
                             offload_enabled=layout.get("g2_blocks", 0) > 0, num_workers=max(1, len(self._workers)),
                             **disagg_leader_kwargs(cfg))
        # operator / peer control plane on the runtime's messenger (describe, reset, metrics)
        import dataclasses
        import json

        from .engine.control import LeaderControl

        plain = json.loads(json.dumps(dataclasses.asdict(cfg), default=str))
        self.control = LeaderControl(self._impl.leader, self.runtime.messenger, self.block_size,
                                     role=(plain.get("disagg") or {}).get("role"), config=plain,
                                     parallelism={"workers": max(1, len(self._workers))},
                                     cd_stats=lambda: self._impl.cd_stats)

    def _need(self) -> _Leader:
        if self._impl is None:
            raise RuntimeError("ConnectorLeader not initialized: call initialize_workers()")
        return self._impl

    def create_slot(self, request: KvbmRequest) -> None:
        self._need().create_slot(request)

    def has_slot(self, request_id: str) -> bool:
        return self._impl is not None and self._impl.has_slot(request_id)

    def get_num_new_matched_tokens(self, request_id: str, num_computed_tokens: int):
        return self._need().get_num_new_matched_tokens(request_id, num_computed_tokens)

    def update_state_after_alloc(self, request_id: str, block_ids: list[int], num_external_tokens: int) -> None:
        self._need().update_state_after_alloc(request_id, block_ids, num_external_tokens)

    def build_connector_metadata(self, output: SchedulerOutput | SchedulerOutputLite) -> bytes:
        lite = output.lite() if isinstance(output, SchedulerOutput) else output
        return self._need().build_connector_meta(lite)

    def update_connector_output(self, finished_sending=None, finished_recving=None) -> None:
        self._need().update_connector_output(finished_sending, finished_recving)

    def request_finished(self, request_id: str):
        return self._need().request_finished(request_id)

    build_connector_meta = build_connector_metadata

    def extend_slot_tokens(self, request_id: str, tokens: list[int]) -> None:
        """Append tokens (e.g. generated ones) to a request's sequence outside a scheduler step."""
        self._need().slots[request_id].seq.append(list(tokens))

    def get_slot_total_tokens(self, request_id: str) -> int:
        return len(self._need().slots[request_id].seq)


class ConnectorWorker:
    """Worker-side connector bound to a runtime; serves its layout to the leader."""

    def __init__(self, runtime: KvbmRuntime, block_size: int = 16, num_kv_heads: int | None = None,
                 head_size: int | None = None, rank: int = 0):
        from .connector.worker import ConnectorWorker as _Worker

        self.runtime, self.rank = runtime, rank
        self._impl = _Worker(runtime.config, rank=rank, block_size=block_size, num_kv_heads=num_kv_heads,
                             head_size=head_size)
        self._service = None
        runtime.messenger.register_handler(LAYOUT_HANDLER, lambda _p: self._impl.handshake_metadata())

    def _serve(self):
        """Once the KV caches are registered, serve this rank's block operations to the leader."""
        from .engine.spmd import WorkerService

        if self._service is None and self._impl.worker is not None:
            self._service = WorkerService(self.runtime.messenger, self._impl.worker, self.rank)

    def register_kv_caches(self, *a, **kw):
        out = self._impl.register_kv_caches(*a, **kw)
        self._serve()
        return out

    def register_cross_layers_kv_cache(self, *a, **kw):
        out = self._impl.register_cross_layers_kv_cache(*a, **kw)
        self._serve()
        return out

    def register_layout(self, layout):
        out = self._impl.register_layout(layout)
        self._serve()
        return out

    # the worker hooks, explicitly (the reference's binding names)
    def bind_connector_metadata(self, metadata: bytes) -> None:
        self._impl.bind_connector_metadata(metadata)

    def clear_connector_metadata(self) -> None:
        self._impl.clear_connector_metadata()

    def start_load_kv(self) -> None:
        self._impl.start_load_kv()

    def wait_for_layer_load(self, layer) -> None:
        self._impl.wait_for_layer_load(layer)

    def save_kv_layer(self, layer, requests=None) -> None:
        self._impl.save_kv_layer(layer, requests)

    def wait_for_save(self) -> None:
        self._impl.wait_for_save()

    def get_finished(self, finished_req_ids=None):
        return self._impl.get_finished(set(finished_req_ids or ()))

    def get_failed_onboarding(self) -> set[int]:
        """G1 block ids whose load failed (the framework recomputes them)."""
        return self._impl.get_block_ids_with_load_errors()

    def handle_preemptions(self, preempted_req_ids) -> None:
        self._impl.handle_preemptions(preempted_req_ids)

    def handshake_metadata(self) -> dict:
        return self._impl.handshake_metadata()

    def is_initialized(self) -> bool:
        return self._impl.worker is not None

    def shutdown(self) -> None:
        self._impl.shutdown()

    def __getattr__(self, name):
        return getattr(self._impl, name)


hub = types.ModuleType("kvbm_b200._core.hub")
hub.PrefillRouterHandler = _hub_client.PrefillRouterHandler
hub.CompletionEvent = _hub_client.CompletionEvent

__all__ = ["KvbmRuntime", "ConnectorLeader", "ConnectorWorker", "KvbmRequest", "SchedulerOutput", "Tensor",
           "KvbmVllmConfig", "is_available", "hub", "__version__"]
