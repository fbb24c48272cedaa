"""vLLM v1 KV-connector adapter (``kv_connector_module_path=kvbm_b200.connector.vllm_connector``,
``kv_connector=KvbmConnector``).

Importing this module does not import vLLM until a connector is built, so
the package stays importable without vLLM (the reference tests the same
lazy-import property: python/tests/test_connector_lazy_import.py).

Role dispatch and hook set follow python/kvbm/vllm/connector/base.py:55-473
(KvbmConnector), leader.py and worker.py; the scheduler process runs a
:class:`~kvbm_b200.connector.leader.ConnectorLeader` over an
:class:`~kvbm_b200.engine.leader.InstanceLeader`, each GPU worker a
:class:`~kvbm_b200.connector.worker.ConnectorWorker`.
"""

from __future__ import annotations

import dataclasses
import json
import os
from typing import Any, Protocol

from .config import extract_vllm_config_for_kvbm, kv_block_bytes
from .leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
from .protocol import ConnectorMetadata


class NewRequestDataProtocol(Protocol):
    """The fields of vLLM's ``NewRequestData`` the connector reads."""

    req_id: str
    prompt_token_ids: list[int] | None
    block_ids: tuple[list[int], ...]
    num_computed_tokens: int


class CachedRequestDataProtocol(Protocol):
    """The fields of vLLM's ``CachedRequestData`` the connector reads (one list entry per request)."""

    req_ids: list[str]
    new_token_ids: list[list[int]]
    new_block_ids: list[tuple[list[int], ...] | None]
    num_computed_tokens: list[int]


class SchedulerOutputProtocol(Protocol):
    """The fields of vLLM's ``SchedulerOutput`` the connector reads."""

    scheduled_new_reqs: list[NewRequestDataProtocol]
    scheduled_cached_reqs: CachedRequestDataProtocol
    num_scheduled_tokens: dict[str, int]
    finished_req_ids: set[str]


def process_scheduler_output(step: int, so, slots: dict) -> SchedulerOutputLite:
    """vLLM SchedulerOutput -> the connector's framework-neutral step view."""
    out = SchedulerOutputLite(step=step)
    sched = dict(getattr(so, "num_scheduled_tokens", {}) or {})
    for nr in getattr(so, "scheduled_new_reqs", []) or []:
        blocks = list(nr.block_ids[0]) if nr.block_ids else []
        slot = slots.get(nr.req_id)
        if slot is not None and slot.g1_block_ids and blocks[: len(slot.g1_block_ids)] == slot.g1_block_ids:
            blocks = blocks[len(slot.g1_block_ids):]  # update_state_after_alloc already recorded these
        out.scheduled[nr.req_id] = ([], blocks, nr.num_computed_tokens + sched.get(nr.req_id, 0))
    cached = getattr(so, "scheduled_cached_reqs", None)
    if cached is not None:
        all_tok = getattr(cached, "all_token_ids", {}) or {}
        for i, rid in enumerate(cached.req_ids):
            nb = cached.new_block_ids[i]
            new_blocks = list(nb[0]) if nb else []
            slot = slots.get(rid)
            toks: list[int] = []
            if slot is not None:
                full = all_tok.get(rid)
                if full is not None:
                    toks = list(full[len(slot.seq):])
                elif cached.new_token_ids and i < len(cached.new_token_ids):
                    toks = list(cached.new_token_ids[i])
            out.scheduled[rid] = (toks, new_blocks, cached.num_computed_tokens[i] + sched.get(rid, 0))
    out.finished_req_ids = list(getattr(so, "finished_req_ids", []) or [])
    out.preempted_req_ids = sorted(getattr(so, "preempted_req_ids", None) or [])
    return out


def disagg_leader_kwargs(cfg) -> dict:
    """ConnectorLeader arguments for the configured disaggregation role (none when unset).

    Every role joins the node's plane as ``disagg.instance_id``: any instance
    accepts remote prefills and pushes their KV to the decode instance named in
    the request's ``kv_transfer_params``. A decode instance also decides per
    request (``disagg.selection``) and sends remote prefills to
    ``disagg.prefill_instance`` over the plane at ``disagg.directory``, or,
    with ``hub.url`` set and no prefill instance named, through the hub's
    prefill router (which then picks the prefill engine)."""
    dis = cfg.disagg
    if dis is None or not dis.role:
        return {}
    if dis.instance_id is None:
        raise ValueError("disagg.role needs disagg.instance_id (the scheduler and its workers share it)")
    from ..engine.cd import ConditionalDisagg, InflightBudget, SelectionPolicy
    from ..engine.cd_plane import HubRouterPlane, open_cd_services

    plane, directory = open_cd_services(dis.directory)
    kw: dict = {"instance_id": int(dis.instance_id), "directory": directory}
    if dis.role in ("decode", "both") and dis.selection != "never":
        slots = int(dis.mailbox_slots)
        kw.update(cd=ConditionalDisagg(SelectionPolicy(dis.selection, dis.min_remote_prefill_tokens),
                                       InflightBudget(dis.max_inflight or slots), fallback=dis.fallback),
                  mailbox_slots=slots, recv_timeout_s=float(dis.recv_timeout_s))
        if dis.prefill_instance is not None:
            kw.update(plane=plane, prefill_target=int(dis.prefill_instance))
        elif cfg.hub is not None and cfg.hub.url:
            from ..hub.client import HubClient

            # the router picks the prefill engine: contributor counts assume its TP degree divides ours
            kw.update(plane=HubRouterPlane(HubClient(cfg.hub.url)), prefill_target=0, directory=None)
        else:
            raise ValueError("disagg decode role needs disagg.prefill_instance or hub.url")
    return kw


def disagg_worker_enable(worker, cfg, tp_rank: int, tp_size: int) -> bool:
    """Join the plane from a model-runner worker once its KV caches are registered: publish
    the pool (through CUDA IPC records of the engine's own KV tensors) and, on a decode
    instance, the mailbox the prefill workers complete into."""
    dis = cfg.disagg
    if dis is None or not dis.role:
        return False
    from ..engine.cd_plane import open_cd_services

    _, directory = open_cd_services(dis.directory)
    receives = dis.role in ("decode", "both") and dis.selection != "never"
    worker.enable_disagg(int(dis.instance_id), directory, mailbox_slots=int(dis.mailbox_slots) if receives else 0,
                         shared=True, tp_rank=tp_rank, tp_size=tp_size)
    return True


def _object_store(cfg):
    """The G4 store the scheduler checks presence in (the workers open their own), or None."""
    if cfg.object is None:
        return None
    from ..object import make_object_store

    return make_object_store(cfg.object)


def instance_id_for(cfg, vllm_config) -> int:
    """This engine's instance id, the same in its scheduler and its workers: ``disagg.instance_id``
    when set, else derived from vLLM's per-engine ``engine_id``."""
    if cfg.disagg is not None and cfg.disagg.instance_id is not None:
        return int(cfg.disagg.instance_id)
    import uuid

    eid = str(getattr(vllm_config.kv_transfer_config, "engine_id", "") or "")
    try:
        return uuid.UUID(eid).int >> 64
    except ValueError:
        return uuid.uuid5(uuid.NAMESPACE_OID, eid or "kvbm").int >> 64


def g2_directory(cfg):
    """Where an engine's workers publish their G2 pool files for remote search (on this node)."""
    import os as _os

    from ..engine.cd_plane import FilePeerDirectory

    url = cfg.disagg.directory if cfg.disagg is not None else "file:///dev/shm/kvbm_pd"
    root = url[len("file://"):] if url.startswith("file://") else "/dev/shm/kvbm_pd"
    return FilePeerDirectory(_os.path.join(root, "g2"))


class RemoteSearchPlane:
    """A scheduler's side of remote search: its messenger (serving its own G2 blocks to other
    instances as a holder), its hub registration and the search itself, whose pulls the
    connector's workers run (``ConnectorLeader.queue_remote_pull``)."""

    def __init__(self, cfg, leader: ConnectorLeader, instance_id: int, tp_size: int, block_size: int):
        from ..engine.remote_search import RemoteHolder, RemoteSearch, RemoteSearchConfig
        from ..hub.client import HubClient, HubRegistration
        from ..runtime.messenger import Messenger

        if cfg.hub is None or not cfg.hub.url:
            raise ValueError("remote_search.enabled needs hub.url (the hub's indexer finds the holders)")
        rs = cfg.remote_search
        self.messenger = Messenger(instance_id)
        self.hub = HubClient(cfg.hub.url)
        self.registration = HubRegistration(self.hub, instance_id, features=["indexer", "p2p"],
                                            address=self.messenger.address)
        g2dir = g2_directory(cfg)
        self.holder = RemoteHolder(leader.leader, [], self.messenger, pool_source=lambda: [
            g2dir.lookup(instance_id, timeout_s=rs.timeout_secs, rank=r) for r in range(tp_size)])
        self.search = RemoteSearch(leader.leader, [], self.messenger, self.hub, block_size,
                                   RemoteSearchConfig(enabled=True, min_remote_tokens=rs.min_remote_tokens,
                                                      max_query_hashes=rs.max_query_hashes, timeout=rs.timeout_secs),
                                   copier=lambda pools, src, dst: leader.queue_remote_pull(
                                       pools, src, dst, timeout=max(30.0, 6 * rs.timeout_secs)))
        leader.remote = self.search

    def close(self) -> None:
        self.search.close()
        self.registration.close()
        self.messenger.close()


def _base():
    from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1, KVConnectorMetadata,
                                                                  KVConnectorRole)
    return KVConnectorBase_V1, KVConnectorMetadata, KVConnectorRole


def __getattr__(name):  # lazily build the vLLM subclasses on first access
    if name in ("KvbmConnector", "KvbmConnectorMetadata", "KvbmConnectorWorkerMetadata"):
        _define()
        return globals()[name]
    raise AttributeError(name)


def _define():
    if "KvbmConnector" in globals():
        return
    Base, MetaBase, Role = _base()

    class KvbmConnectorMetadata(MetaBase):
        def __init__(self, metadata: bytes):
            assert isinstance(metadata, bytes)
            self.metadata = metadata

    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorWorkerMetadata as WorkerMetaBase
    except ImportError:  # older vLLM: no worker -> scheduler channel
        WorkerMetaBase = object

    class KvbmConnectorWorkerMetadata(WorkerMetaBase):
        """Worker -> scheduler report: steps whose G1 -> G2 copies / G2 -> G3 spills and remote pulls a
        worker finished, summed over workers."""

        def __init__(self, data: dict):
            self.data = data

        def aggregate(self, other):
            # every report kind (offloaded / spilled steps, pulled ids) maps an id to a worker count
            out: dict = {}
            for d in (self.data, other.data):
                for kind, counts in (d or {}).items():
                    m = out.setdefault(kind, {})
                    for k, v in counts.items():
                        m[int(k)] = m.get(int(k), 0) + int(v)
            return KvbmConnectorWorkerMetadata(out)

    class KvbmConnector(Base):
        """KV Block Manager connector for vLLM (scheduler and worker roles)."""

        def __init__(self, vllm_config, role, kv_cache_config=None):
            super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)
            from ..engine.leader import InstanceLeader
            from ..logical.manager import BlockManager, Tier
            from ..utils.config import KvbmConfig
            from .worker import ConnectorWorker, blocks_for_bytes

            ktc = vllm_config.kv_transfer_config
            self._vllm_config = vllm_config
            extra = getattr(ktc, "kv_connector_extra_config", {}) or {}
            self.info = extract_vllm_config_for_kvbm(vllm_config)
            bs = self.info["block_size"]
            self._step = 0
            if role == Role.SCHEDULER:
                cfg = KvbmConfig.for_leader(json.dumps(extra) if extra else None)
                bpb = kv_block_bytes(self.info)
                g2n = blocks_for_bytes(cfg.cache.host.cache_size_gb, cfg.cache.host.num_blocks, bpb)
                g3n = blocks_for_bytes(cfg.cache.disk.cache_size_gb, cfg.cache.disk.num_blocks, bpb)
                from .consolidator_config import get_consolidator_endpoints

                # the G2/G3 presence events go to the configured sink (events.enabled), to the KV-event
                # consolidator (merged with vLLM's G1 events) and, with remote search, to the hub's indexer
                self.consolidator = self._events = None
                eps = get_consolidator_endpoints(vllm_config)
                iid = instance_id_for(cfg, vllm_config)
                searching = bool(cfg.remote_search.enabled)
                if eps is not None or cfg.events.enabled or searching:
                    from ..logical.events import HubEventSink, events_from_config

                    ev_cfg = cfg.events if cfg.events.enabled else dataclasses.replace(cfg.events, endpoint=None)
                    self._events = events_from_config(ev_cfg, iid, cfg.hub.url if cfg.hub else None)
                    if searching and ev_cfg.endpoint != "hub" and cfg.hub is not None and cfg.hub.url:
                        from ..hub.client import HubClient

                        self._events.add_sink(HubEventSink(HubClient(cfg.hub.url)))  # holders for the indexer
                if eps is not None:
                    from ..consolidator.service import start_leader_consolidator

                    self.consolidator = start_leader_consolidator(eps[0], eps[1], "vllm", bs, self._events)
                if self._events is not None:
                    self._events.start()
                # offload policies from the configuration; an access-frequency sketch when one needs it
                from .. import _core_native as core
                from ..engine.offload import make_policy

                pol = cfg.offload
                lfu = any("lfu" in p for p in pol.g1_to_g2.policies + pol.g2_to_g3.policies)
                g2 = BlockManager(max(1, g2n), bs, cfg.cache.inactive_backend, Tier.G2,
                                  duplicate_policy=cfg.cache.duplicate_policy,
                                  events=self._events.queue if self._events is not None else None,
                                  frequency=core.TinyLfu() if lfu and cfg.cache.inactive_backend != "multi_lru"
                                  else None)
                g3 = BlockManager(g3n, bs, cfg.cache.inactive_backend, Tier.G3, registry=g2.registry) if g3n else None
                decode_offload = os.getenv("KVBM_DECODE_OFFLOAD")
                self._leader = ConnectorLeader(InstanceLeader.scheduler_side(g2, g3), bs,
                                               offload_enabled=g2n > 0,
                                               decode_offload=(pol.decode_offload if decode_offload is None
                                                               else decode_offload == "true"),
                                               g2_policy=make_policy(pol.g1_to_g2.policies, g2),
                                               g3_policy=make_policy(pol.g2_to_g3.policies, g3) if g3 is not None
                                               else None,
                                               num_workers=max(1, int(self.info.get("tensor_parallel_size", 1))),
                                               tp_size=max(1, int(self.info.get("tensor_parallel_size", 1))),
                                               objects=_object_store(cfg), **disagg_leader_kwargs(cfg))
                self._metrics_server = None
                if cfg.metrics.enabled:
                    # Prometheus endpoint of the scheduler: pool occupancy, matches, cache hit rates
                    from ..utils.metrics import KvbmCollector, serve_metrics

                    col = KvbmCollector()
                    col.add_pool("g2", g2)
                    if g3 is not None:
                        col.add_pool("g3", g3)
                    col.cache = self._leader.stats
                    if self._leader.cd is not None:
                        self._leader.cd.metrics = col.cd  # kvbm_cd_* counters from the decisions
                    self._metrics_server = serve_metrics(col, int(cfg.metrics.port))
                self._remote = None
                if searching:
                    self._remote = RemoteSearchPlane(cfg, self._leader, iid,
                                                     max(1, int(self.info.get("tensor_parallel_size", 1))), bs)
                self._worker = None
            else:
                cfg = KvbmConfig.for_worker(json.dumps(extra) if extra else None)
                self._worker = ConnectorWorker(cfg, rank=self.info.get("rank", 0), block_size=bs,
                                               num_kv_heads=self.info["num_kv_heads"],
                                               head_size=self.info["head_size"])
                self._leader = None
            self._cfg = cfg

        # ------------------------------------------------ scheduler side
        @property
        def prefer_cross_layer_blocks(self) -> bool:
            return os.getenv("KVBM_PREFER_FULLY_CONTIGUOUS_BLOCKS", "false") == "true"

        def _slot(self, request):
            if not self._leader.has_slot(request.request_id):
                salt = getattr(request, "cache_salt", None)
                lora = getattr(getattr(request, "lora_request", None), "lora_name", None)
                self._leader.create_slot(KvbmRequest(request.request_id, list(request.prompt_token_ids),
                                                     lora_name=lora, salt=salt,
                                                     kv_transfer_params=getattr(request, "kv_transfer_params",
                                                                                None)))

        def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
            self._slot(request)
            return self._leader.get_num_new_matched_tokens(request.request_id, num_computed_tokens)

        def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
            self._slot(request)
            ids = [int(b) for b in blocks.get_block_ids()[0]]
            self._leader.update_state_after_alloc(request.request_id, ids, num_external_tokens)

        def build_connector_meta(self, scheduler_output):
            self._step += 1
            lite = process_scheduler_output(self._step, scheduler_output, self._leader.slots)
            return KvbmConnectorMetadata(self._leader.build_connector_meta(lite))

        def update_connector_output(self, connector_output):
            wm = getattr(connector_output, "kv_connector_worker_meta", None)
            self._leader.update_connector_output(getattr(connector_output, "finished_sending", None),
                                                 getattr(connector_output, "finished_recving", None),
                                                 getattr(wm, "data", None),
                                                 getattr(connector_output, "invalid_block_ids", None))

        def request_finished(self, request, block_ids):
            return self._leader.request_finished(request.request_id, list(block_ids))

        def build_kv_connector_stats(self, data=None):
            return None

        # --------------------------------------------------- worker side
        def _join_plane(self):
            tp = max(1, int(self.info.get("tensor_parallel_size", 1)))
            disagg_worker_enable(self._worker, self._cfg, int(self.info.get("rank", 0)) % tp, tp)
            if self._cfg.remote_search.enabled and getattr(self._worker.worker, "g2_layout", None) is not None:
                self._worker.tp_rank, self._worker.tp_size = int(self.info.get("rank", 0)) % tp, tp
                self._worker.publish_g2(g2_directory(self._cfg), instance_id_for(self._cfg, self._vllm_config))

        def register_kv_caches(self, kv_caches):
            self._worker.register_kv_caches(dict(kv_caches))
            self._join_plane()

        def register_cross_layers_kv_cache(self, kv_cache, attn_backend=None):
            self._worker.register_cross_layers_kv_cache(kv_cache)
            self._join_plane()

        def bind_connector_metadata(self, connector_metadata):
            super().bind_connector_metadata(connector_metadata)
            self._worker.bind_connector_metadata(connector_metadata.metadata)

        def clear_connector_metadata(self):
            super().clear_connector_metadata()
            self._worker.clear_connector_metadata()

        def handle_preemptions(self, kv_connector_metadata):
            # before the preempted requests' G1 blocks are overwritten: wait for their offloads
            raw = getattr(kv_connector_metadata, "metadata", None)
            if raw:
                self._worker.handle_preemptions(ConnectorMetadata.decode(raw).evict)

        def start_load_kv(self, forward_context, **kwargs: Any) -> None:
            self._worker.start_load_kv()

        def wait_for_layer_load(self, layer_name: str) -> None:
            self._worker.wait_for_layer_load(layer_name)

        def save_kv_layer(self, layer_name, kv_layer, attn_metadata, **kwargs) -> None:
            self._worker.save_kv_layer(layer_name)

        def wait_for_save(self):
            self._worker.wait_for_save()

        def get_finished(self, finished_req_ids):
            sending, recving = self._worker.get_finished(set(finished_req_ids))
            return (sending or None), (recving or None)

        def get_block_ids_with_load_errors(self):
            return self._worker.get_block_ids_with_load_errors()

        def build_connector_worker_meta(self):
            data = self._worker.build_connector_worker_meta()
            return KvbmConnectorWorkerMetadata(data) if data else None

        def shutdown(self):
            if self._worker is not None:
                self._worker.shutdown()
            if getattr(self, "_events", None) is not None:
                self._events.stop()
            if getattr(self, "consolidator", None) is not None:
                self.consolidator.close()
            if getattr(self, "_remote", None) is not None:
                self._remote.close()
            srv = getattr(self, "_metrics_server", None)
            if srv is not None and isinstance(srv, tuple):
                srv[0].shutdown()  # (server, thread) from prometheus_client

    globals()["KvbmConnector"] = KvbmConnector
    globals()["KvbmConnectorMetadata"] = KvbmConnectorMetadata
    globals()["KvbmConnectorWorkerMetadata"] = KvbmConnectorWorkerMetadata
