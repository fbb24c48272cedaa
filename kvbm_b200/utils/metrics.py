"""Prometheus metrics for the block manager.

Counters live where the work happens (the C++ pools keep atomics; transfer
and disaggregation code increment Python counters); a custom collector reads
them at scrape time, so the hot paths never touch the Prometheus registry.

Metric names follow the reference (crates/kvbm-observability/src/{pool,
collector,transfer,cd,cache}.rs): kvbm_allocations_total,
kvbm_evictions_total, kvbm_registrations_total, kvbm_registration_dedup_total,
kvbm_match_hashes_requested_total, kvbm_match_blocks_returned_total,
kvbm_matched_tokens_total, kvbm_host_cache_hit_rate,
kvbm_disk_cache_hit_rate, kvbm_object_cache_hit_rate,
kvbm_inactive_pool_size, kvbm_reset_pool_size, kvbm_inflight_mutable,
kvbm_inflight_immutable, kvbm_transfer_duration_seconds,
kvbm_transfer_inflight, kvbm_transfer_failures_total, kvbm_cd_*.

``StatsCollector`` turns one pool's cumulative counters into a rolling window
of derived figures (allocation and eviction rates per second and their
change per second, match and scan hit ratios over the interval, pool
occupancy), sampled on demand or by a daemon thread (parity:
crates/kvbm-observability/src/stats.rs:18-200).
"""

from __future__ import annotations

import threading
import time
from collections import deque
from dataclasses import dataclass

from prometheus_client import CollectorRegistry, start_http_server
from prometheus_client.core import CounterMetricFamily, GaugeMetricFamily, HistogramMetricFamily


class TransferMetrics:
    BUCKETS = (1e-4, 5e-4, 1e-3, 5e-3, 1e-2, 5e-2, 0.1, 0.5, 1.0, 5.0)

    def __init__(self):
        self._lock = threading.Lock()
        self.inflight = 0
        self.failures = 0
        self.bytes = 0
        self.counts = [0] * (len(self.BUCKETS) + 1)
        self.sum = 0.0

    def observe(self, seconds: float, nbytes: int = 0) -> None:
        with self._lock:
            self.sum += seconds
            self.bytes += nbytes
            for i, b in enumerate(self.BUCKETS):
                if seconds <= b:
                    self.counts[i] += 1
                    break
            else:
                self.counts[-1] += 1

    def start(self) -> None:
        with self._lock:
            self.inflight += 1

    def finish(self, ok: bool = True) -> None:
        with self._lock:
            self.inflight -= 1
            if not ok:
                self.failures += 1


class CacheStatsTracker:
    """Sliding-window hit rate per tier over the last N requests."""

    def __init__(self, max_requests: int = 1000):
        self._win: dict[str, deque] = {}
        self.max_requests = max_requests
        self.matched_tokens = 0
        self._lock = threading.Lock()

    def record(self, tier: str, requested_blocks: int, hit_blocks: int, block_size: int = 16) -> None:
        with self._lock:
            d = self._win.setdefault(tier, deque(maxlen=self.max_requests))
            d.append((requested_blocks, hit_blocks))
            self.matched_tokens += hit_blocks * block_size

    def hit_rate(self, tier: str) -> float:
        with self._lock:
            d = self._win.get(tier)
            if not d:
                return 0.0
            req = sum(r for r, _ in d)
            return sum(h for _, h in d) / req if req else 0.0


class CdMetrics:
    def __init__(self):
        self.decisions = {"local": 0, "remote": 0, "fallback": 0}
        self.remote_tokens = 0
        self.breaker_tier = 0


class KvbmCollector:
    """Reads pool/transfer/cache/cd counters at scrape time."""

    def __init__(self):
        self.pools: dict[str, object] = {}  # tier name -> BlockManager
        self.transfer = TransferMetrics()
        self.cache = CacheStatsTracker()
        self.cd = CdMetrics()

    def add_pool(self, tier: str, manager) -> None:
        self.pools[tier] = manager

    def collect(self):
        counters = {
            "allocations": "kvbm_allocations_total",
            "evictions": "kvbm_evictions_total",
            "registrations": "kvbm_registrations_total",
            "registration_dedup": "kvbm_registration_dedup_total",
            "match_hashes_requested": "kvbm_match_hashes_requested_total",
            "match_blocks_returned": "kvbm_match_blocks_returned_total",
        }
        fams = {k: CounterMetricFamily(v[: -len("_total")], f"kvbm {k}", labels=["tier"]) for k, v in
                counters.items()}
        inactive = GaugeMetricFamily("kvbm_inactive_pool_size", "inactive (evictable) blocks", labels=["tier"])
        reset = GaugeMetricFamily("kvbm_reset_pool_size", "reset (free) blocks", labels=["tier"])
        inflight = GaugeMetricFamily("kvbm_inflight_immutable", "registered blocks in use", labels=["tier"])
        for tier, mgr in self.pools.items():
            m = mgr.metrics()
            for k, fam in fams.items():
                fam.add_metric([tier], m.get(k, 0))
            inactive.add_metric([tier], mgr.inactive_len())
            reset.add_metric([tier], mgr.reset_len())
            inflight.add_metric([tier], mgr.active_len())
        yield from fams.values()
        yield inactive
        yield reset
        yield inflight
        mt = CounterMetricFamily("kvbm_matched_tokens", "tokens matched from the cache")
        mt.add_metric([], self.cache.matched_tokens)
        yield mt
        for tier, name in (("host", "kvbm_host_cache_hit_rate"), ("disk", "kvbm_disk_cache_hit_rate"),
                           ("object", "kvbm_object_cache_hit_rate")):
            g = GaugeMetricFamily(name, f"{tier} cache hit rate (sliding window)")
            g.add_metric([], self.cache.hit_rate(tier))
            yield g
        t = self.transfer
        h = HistogramMetricFamily("kvbm_transfer_duration_seconds", "transfer duration")
        acc, buckets = 0, []
        for b, c in zip(list(t.BUCKETS) + [float("inf")], t.counts):
            acc += c
            buckets.append((str(b) if b != float("inf") else "+Inf", acc))
        h.add_metric([], buckets, t.sum)
        yield h
        g = GaugeMetricFamily("kvbm_transfer_inflight", "transfers in flight")
        g.add_metric([], t.inflight)
        yield g
        c = CounterMetricFamily("kvbm_transfer_failures", "failed transfers")
        c.add_metric([], t.failures)
        yield c
        d = CounterMetricFamily("kvbm_cd_decisions", "conditional-disagg decisions", labels=["decision"])
        for k, v in self.cd.decisions.items():
            d.add_metric([k], v)
        yield d
        rt = CounterMetricFamily("kvbm_cd_remote_prefill_tokens", "tokens prefilled remotely")
        rt.add_metric([], self.cd.remote_tokens)
        yield rt
        bt = GaugeMetricFamily("kvbm_cd_breaker_tier", "prefill-router breaker tier (0 calm, 1 warm, 2 hot)")
        bt.add_metric([], self.cd.breaker_tier)
        yield bt


@dataclass(frozen=True)
class StatsSnapshot:
    allocation_rate: float = 0.0      # blocks allocated per second over the last interval
    eviction_rate: float = 0.0
    match_hit_rate: float = 0.0       # blocks returned / hashes requested by prefix matches in the interval
    scan_hit_rate: float = 0.0
    allocation_gradient: float = 0.0  # change of allocation_rate per second
    eviction_gradient: float = 0.0
    inflight_mutable: int = 0
    inflight_immutable: int = 0
    reset_pool_size: int = 0
    inactive_pool_size: int = 0


class StatsCollector:
    """Rolling window of derived pool statistics. Disabled until ``set_enabled(True)``; ``sample``
    is then cheap (one counter read) and may be called from any thread."""

    def __init__(self, manager, window_size: int = 60, sample_interval_s: float = 1.0, clock=time.monotonic):
        self.mgr = manager
        self.window_size, self.interval = int(window_size), float(sample_interval_s)
        self._clock = clock
        self._enabled = False
        self._entries: deque = deque(maxlen=self.window_size)
        self._lock = threading.Lock()
        self._thread: threading.Thread | None = None
        self._stop = threading.Event()

    def set_enabled(self, on: bool) -> None:
        self._enabled = bool(on)

    def is_enabled(self) -> bool:
        return self._enabled

    def _raw(self) -> dict:
        m = dict(self.mgr.metrics())
        m["inflight_immutable"] = self.mgr.active_len()
        m["reset_pool_size"] = self.mgr.reset_len()
        m["inactive_pool_size"] = self.mgr.inactive_len()
        m["inflight_mutable"] = max(0, self.mgr.total_blocks() - m["inflight_immutable"] - m["reset_pool_size"]
                                    - m["inactive_pool_size"])
        return m

    def sample(self) -> StatsSnapshot | None:
        if not self._enabled:
            return None
        now, raw = self._clock(), self._raw()
        occ = {k: raw[k] for k in ("inflight_mutable", "inflight_immutable", "reset_pool_size", "inactive_pool_size")}
        with self._lock:
            prev = self._entries[-1] if self._entries else None
            dt = now - prev[0] if prev else 0.0
            if prev is None or dt <= 0:
                st = StatsSnapshot(**occ)
            else:
                p, ps = prev[1], prev[2]

                def ratio(req, ret):
                    dq = raw[req] - p[req]
                    return (raw[ret] - p[ret]) / dq if dq > 0 else 0.0

                ar = (raw["allocations"] - p["allocations"]) / dt
                er = (raw["evictions"] - p["evictions"]) / dt
                st = StatsSnapshot(ar, er, ratio("match_hashes_requested", "match_blocks_returned"),
                                   ratio("scan_hashes_requested", "scan_blocks_returned"),
                                   (ar - ps.allocation_rate) / dt, (er - ps.eviction_rate) / dt, **occ)
            self._entries.append((now, raw, st))
        return st

    def latest(self) -> StatsSnapshot | None:
        with self._lock:
            return self._entries[-1][2] if self._entries else None

    def window(self, n: int) -> list[StatsSnapshot]:
        """The last ``n`` snapshots, oldest first."""
        with self._lock:
            return [e[2] for e in list(self._entries)[-n:]] if n > 0 else []

    def spawn(self) -> threading.Thread:
        """Sample every ``sample_interval_s`` on a daemon thread until ``stop``."""
        def loop():
            while not self._stop.wait(self.interval):
                self.sample()
        self._thread = threading.Thread(target=loop, name="kvbm-stats", daemon=True)
        self._thread.start()
        return self._thread

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)


def make_registry(collector: KvbmCollector) -> CollectorRegistry:
    reg = CollectorRegistry()
    reg.register(collector)
    return reg


def serve_metrics(collector: KvbmCollector, port: int, addr: str = "127.0.0.1"):
    """Start the /metrics HTTP endpoint (KVBM_METRICS_PORT)."""
    return start_http_server(port, addr=addr, registry=make_registry(collector))


class Timer:
    def __init__(self, metrics: TransferMetrics, nbytes: int = 0):
        self.m, self.nbytes = metrics, nbytes

    def __enter__(self):
        self.t0 = time.perf_counter()
        self.m.start()
        return self

    def __exit__(self, et, ev, tb):
        self.m.finish(ok=et is None)
        self.m.observe(time.perf_counter() - self.t0, self.nbytes)
