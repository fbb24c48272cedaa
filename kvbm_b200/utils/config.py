"""Layered configuration (``KvbmConfig``).

Precedence, lowest to highest:

1. code defaults (the dataclasses below);
2. legacy ``DYN_KVBM_*`` environment variables (v1 names mapped to paths);
3. ``/opt/dynamo/etc/kvbm.toml``;
4. the TOML file named by ``$KVBM_CONFIG_PATH``;
5. ``KVBM_*`` environment variables: ``KVBM_<SECTION>_<KEY>`` with ``__``
   separating nested levels (``KVBM_CACHE_HOST__CACHE_SIZE_GB=8``) and a
   table of documented short names (``KVBM_CACHE_HOST_SIZE_GB``, ...);
6. a JSON override (vLLM's ``kv_transfer_config.kv_connector_extra_config``)
   with optional ``default`` / ``leader`` / ``worker`` profile sections.

Parity: crates/kvbm-config/src/lib.rs:96-300 (KvbmConfig, figment layering,
leader/worker profiles), cache.rs (ParallelismMode, host/disk sizes),
offload.rs, onboard.rs (OnboardMode), disagg.rs, events.rs, metrics.rs,
v1_compat.rs (DYN_KVBM_* mapping).
"""

from __future__ import annotations

import copy
import dataclasses
import json
import os
import tomllib
from dataclasses import dataclass, field
from typing import Any

SYSTEM_TOML = "/opt/dynamo/etc/kvbm.toml"


@dataclass
class HostCacheConfig:
    cache_size_gb: float | None = None
    num_blocks: int | None = None
    # NUMA placement of the G2 pool: None (cudaHostAlloc decides), "gpu" (the node nearest
    # to the worker's GPU) or a node number; optionally on 2 MiB huge pages
    numa_node: int | str | None = None
    hugepages: bool = False


@dataclass
class DiskCacheConfig:
    cache_size_gb: float | None = None
    num_blocks: int | None = None
    dir: str | None = None
    use_direct_io: bool = True
    persistent: bool = False


@dataclass
class CacheConfig:
    host: HostCacheConfig = field(default_factory=HostCacheConfig)
    disk: DiskCacheConfig = field(default_factory=DiskCacheConfig)
    parallelism: str = "tensor_parallel"   # tensor_parallel | replicated_data
    bypass_host_cache: bool = False
    inactive_backend: str = "lineage"      # lineage | lru | multi_lru | lineage_fifo
    duplicate_policy: str = "allow"

    def validate(self) -> None:
        if self.parallelism not in ("tensor_parallel", "replicated_data"):
            raise ValueError(f"cache.parallelism: {self.parallelism!r}")


@dataclass
class PipelineConfig:
    policies: list[str] = field(default_factory=lambda: ["presence"])
    max_batch: int = 64
    min_batch: int = 8
    flush_ms: float = 10.0
    policy_timeout_ms: float = 100.0
    sweep_ms: float = 10.0
    concurrency: int = 1


@dataclass
class OffloadConfig:
    g1_to_g2: PipelineConfig = field(default_factory=PipelineConfig)
    g2_to_g3: PipelineConfig = field(default_factory=lambda: PipelineConfig(policies=["presence_lfu"]))
    g2_to_g4: PipelineConfig = field(default_factory=lambda: PipelineConfig(policies=["object_presence"]))
    decode_offload: bool = False


@dataclass
class OnboardConfig:
    mode: str = "inter"   # inter (between passes) | intra (layer-wise inside the pass)


@dataclass
class ObjectConfig:
    bucket: str = "kvbm"
    kind: str = "fs"             # fs (a directory standing in for a bucket) | s3 (S3 REST API, SigV4)
    root: str | None = None      # filesystem-backed store root
    endpoint: str | None = None  # S3 endpoint URL (MinIO, RGW); None: AWS for `region`
    region: str = "us-east-1"
    force_path_style: bool = True
    max_concurrent_requests: int = 16
    lock: bool = True


@dataclass
class EventsConfig:
    enabled: bool = False
    policy: str = "power_of_two"   # power_of_two | all
    min_position: int = 16
    max_position: int = 65536
    window_ms: float = 10.0
    max_batch: int = 1024
    endpoint: str | None = None


@dataclass
class MetricsConfig:
    enabled: bool = False
    port: int = 6880
    cache_stats_max_requests: int = 1000
    cache_stats_log_interval_secs: float = 5.0


@dataclass
class DebugConfig:
    recording: bool = False


@dataclass
class HubConfig:
    url: str | None = None
    heartbeat_secs: float = 5.0
    features: list[str] = field(default_factory=list)  # hub features this connector takes part in


@dataclass
class DisaggSettings:
    role: str | None = None            # prefill | decode | both
    selection: str = "never"           # never | always | threshold
    min_remote_prefill_tokens: int = 512
    max_inflight: int | None = None
    fallback: str = "local"
    drain_poll_ms: float = 2.0
    watchdog_secs: float = 10.0
    # the on-node data plane of remote prefills (a vLLM engine's connector reads these):
    instance_id: int | None = None     # this engine's id on the plane (scheduler and workers agree on it)
    prefill_instance: int | None = None  # decode: where its remote prefills go (a hub routes when unset)
    directory: str = "file:///dev/shm/kvbm_pd"  # file:///path | store://host:port (pools, mailboxes, plane)
    mailbox_slots: int = 64            # decode: remote prefills in flight (one completion word each)
    recv_timeout_s: float = 120.0      # decode: a remote prefill not landed by then is recomputed


@dataclass
class RemoteSearchSettings:
    enabled: bool = False
    min_remote_tokens: int | None = None   # None: any remote match (one block)
    max_query_hashes: int = 64
    timeout_secs: float = 10.0


@dataclass
class MessengerConfig:
    bind: str = "tcp://127.0.0.1:0"        # ZeroMQ endpoint of this instance's RPC server
    discovery: str = "hub"                 # hub | static
    peers: dict = field(default_factory=dict)  # static discovery: instance id -> address


@dataclass
class TransferConfig:
    engine: str = "auto"               # auto | tile | tma | pairs | ce
    max_ctas: int = 0
    allow_gds: bool = False
    allow_gpu_rdma: bool = False
    cuda_graph_replay: bool = False
    startup_benchmark: bool = False
    layer_batch: int = 8               # P->D push: layers per transfer launch during the prefill pass
    push_engine: str = "tma"           # P->D push kernel: tma (bulk-copy pipeline) | tile
    # same-layout pushes into a peer GPU's pool: TMA loads and TMA bulk stores over NVLink (no SM
    # instruction touches the data); false: TMA loads, stores by the consumer warps
    push_bulk_peer: bool = True


@dataclass
class KvbmConfig:
    cache: CacheConfig = field(default_factory=CacheConfig)
    offload: OffloadConfig = field(default_factory=OffloadConfig)
    onboard: OnboardConfig = field(default_factory=OnboardConfig)
    object: ObjectConfig | None = None
    events: EventsConfig = field(default_factory=EventsConfig)
    metrics: MetricsConfig = field(default_factory=MetricsConfig)
    debug: DebugConfig = field(default_factory=DebugConfig)
    hub: HubConfig | None = None
    disagg: DisaggSettings | None = None
    transfer: TransferConfig = field(default_factory=TransferConfig)
    remote_search: RemoteSearchSettings = field(default_factory=RemoteSearchSettings)
    messenger: MessengerConfig = field(default_factory=MessengerConfig)
    max_seq_len: int | None = None
    block_layout: str = "operational"   # operational | universal
    block_size: int = 16

    def validate(self) -> "KvbmConfig":
        self.cache.validate()
        if self.block_layout not in ("operational", "universal"):
            raise ValueError(f"block_layout: {self.block_layout!r}")
        if self.onboard.mode not in ("inter", "intra"):
            raise ValueError(f"onboard.mode: {self.onboard.mode!r}")
        if self.block_size <= 0 or self.block_size & (self.block_size - 1):
            raise ValueError("block_size must be a power of two")
        return self

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    # ----------------------------------------------------------- building
    @classmethod
    def load(cls, json_override: str | dict | None = None, role: str | None = None,
             env: dict[str, str] | None = None, system_toml: str | None = SYSTEM_TOML) -> "KvbmConfig":
        env = dict(os.environ if env is None else env)
        data: dict[str, Any] = {}
        _merge(data, _v1_env(env))
        if system_toml and os.path.exists(system_toml):
            _merge(data, _read_toml(system_toml))
        path = env.get("KVBM_CONFIG_PATH")
        if path:
            _merge(data, _read_toml(path))
        _merge(data, _kvbm_env(env))
        if json_override:
            j = json.loads(json_override) if isinstance(json_override, str) else copy.deepcopy(json_override)
            profiles = {k: j.pop(k) for k in ("default", "leader", "worker") if isinstance(j.get(k), dict)}
            _merge(data, profiles.get("default", {}))
            _merge(data, j)
            if role in ("leader", "worker"):
                _merge(data, profiles.get(role, {}))
        return _build(cls, data).validate()

    @classmethod
    def for_leader(cls, json_override=None, **kw) -> "KvbmConfig":
        return cls.load(json_override, role="leader", **kw)

    @classmethod
    def for_worker(cls, json_override=None, **kw) -> "KvbmConfig":
        return cls.load(json_override, role="worker", **kw)


# --------------------------------------------------------------- helpers

V1_ENV = {
    "DYN_KVBM_CPU_CACHE_GB": "cache.host.cache_size_gb",
    "DYN_KVBM_CPU_CACHE_OVERRIDE_NUM_BLOCKS": "cache.host.num_blocks",
    "DYN_KVBM_DISK_CACHE_GB": "cache.disk.cache_size_gb",
    "DYN_KVBM_DISK_CACHE_OVERRIDE_NUM_BLOCKS": "cache.disk.num_blocks",
    "DYN_KVBM_DISK_CACHE_DIR": "cache.disk.dir",
    "DYN_KVBM_METRICS": "metrics.enabled",
    "DYN_KVBM_METRICS_PORT": "metrics.port",
    "DYN_KVBM_CACHE_STATS_MAX_REQUESTS": "metrics.cache_stats_max_requests",
    "DYN_KVBM_CACHE_STATS_LOG_INTERVAL_SECS": "metrics.cache_stats_log_interval_secs",
    "DYN_KVBM_ENABLE_RECORD": "debug.recording",
    "DYN_KVBM_KV_EVENTS_ENABLE_CONSOLIDATOR": "events.enabled",
    "DYN_KVBM_MAX_TRANSFER_BATCH_SIZE": "offload.g1_to_g2.max_batch",
}

SHORT_ENV = {
    "KVBM_CACHE_HOST_SIZE_GB": "cache.host.cache_size_gb",
    "KVBM_CACHE_HOST_NUM_BLOCKS": "cache.host.num_blocks",
    "KVBM_CACHE_HOST_NUMA_NODE": "cache.host.numa_node",
    "KVBM_CACHE_HOST_HUGEPAGES": "cache.host.hugepages",
    "KVBM_CACHE_DISK_SIZE_GB": "cache.disk.cache_size_gb",
    "KVBM_CACHE_DISK_NUM_BLOCKS": "cache.disk.num_blocks",
    "KVBM_CACHE_DISK_DIR": "cache.disk.dir",
    "KVBM_CACHE_PARALLELISM": "cache.parallelism",
    "KVBM_CACHE_INACTIVE_BACKEND": "cache.inactive_backend",
    "KVBM_OFFLOAD_G1_TO_G2_MAX_BATCH": "offload.g1_to_g2.max_batch",
    "KVBM_OFFLOAD_G1_TO_G2_POLICIES": "offload.g1_to_g2.policies",
    "KVBM_ONBOARD_MODE": "onboard.mode",
    "KVBM_EVENTS_ENABLED": "events.enabled",
    "KVBM_EVENTS_POLICY": "events.policy",
    "KVBM_METRICS_ENABLED": "metrics.enabled",
    "KVBM_METRICS_PORT": "metrics.port",
    "KVBM_BLOCK_LAYOUT": "block_layout",
    "KVBM_BLOCK_SIZE": "block_size",
    "KVBM_TRANSFER_ENGINE": "transfer.engine",
    "KVBM_HUB_URL": "hub.url",
    "KVBM_MAX_SEQ_LEN": "max_seq_len",
    "KVBM_REMOTE_SEARCH_ENABLED": "remote_search.enabled",
    "KVBM_REMOTE_SEARCH_MIN_REMOTE_TOKENS": "remote_search.min_remote_tokens",
    "KVBM_MESSENGER_BIND": "messenger.bind",
}


def _set_path(d: dict, path: str, value) -> None:
    keys = path.split(".")
    for k in keys[:-1]:
        d = d.setdefault(k, {})
    d[keys[-1]] = value


def _parse_scalar(v: str):
    lv = v.strip().lower()
    if lv in ("true", "1", "yes", "on"):
        return True if lv in ("true", "yes", "on") else 1
    if lv in ("false", "no", "off"):
        return False
    for t in (int, float):
        try:
            return t(v)
        except ValueError:
            pass
    if "," in v:
        return [x.strip() for x in v.split(",") if x.strip()]
    return v


def _v1_env(env) -> dict:
    out: dict = {}
    for k, path in V1_ENV.items():
        if k in env:
            _set_path(out, path, _parse_scalar(env[k]))
    if env.get("DYN_KVBM_NCCL_MLA_MODE", "").lower() in ("1", "true"):
        _set_path(out, "cache.parallelism", "replicated_data")
    if env.get("DYN_KVBM_DISABLE_DISK_OFFLOAD_FILTER", "").lower() in ("1", "true"):
        _set_path(out, "offload.g2_to_g3.policies", ["pass_all"])
    return out


def _kvbm_env(env) -> dict:
    out: dict = {}
    for k, v in env.items():
        if not k.startswith("KVBM_") or k in ("KVBM_CONFIG_PATH",):
            continue
        if k in SHORT_ENV:
            _set_path(out, SHORT_ENV[k], _parse_scalar(v))
        elif "__" in k:
            parts = k[len("KVBM_"):].lower().split("__")
            head = parts[0].split("_", 1)
            path = head + parts[1:]
            _set_path(out, ".".join(path), _parse_scalar(v))
    return out


def _read_toml(path: str) -> dict:
    with open(path, "rb") as f:
        return tomllib.load(f)


def _merge(base: dict, over: dict) -> dict:
    for k, v in over.items():
        if isinstance(v, dict) and isinstance(base.get(k), dict):
            _merge(base[k], v)
        else:
            base[k] = copy.deepcopy(v)
    return base


def _build(cls, data: dict):
    if not dataclasses.is_dataclass(cls):
        return data
    kwargs = {}
    hints = {f.name: f for f in dataclasses.fields(cls)}
    for k, v in data.items():
        if k not in hints:
            raise ValueError(f"unknown config key {k!r} in {cls.__name__}")
        f = hints[k]
        sub = _dataclass_of(f.type)
        if sub is not None and isinstance(v, dict):
            kwargs[k] = _build(sub, v)
        else:
            kwargs[k] = v
    return cls(**kwargs)


def _dataclass_of(tp):
    names = {c.__name__: c for c in (HostCacheConfig, DiskCacheConfig, CacheConfig, PipelineConfig, OffloadConfig,
                                     OnboardConfig, ObjectConfig, EventsConfig, MetricsConfig, DebugConfig,
                                     HubConfig, DisaggSettings, TransferConfig, RemoteSearchSettings,
                                     MessengerConfig)}
    s = tp if isinstance(tp, str) else getattr(tp, "__name__", str(tp))
    for name, c in names.items():
        if name in s.replace("None", "").replace("|", " ").split():
            return c
    return None
