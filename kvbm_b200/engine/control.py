"""Leader control plane: typed request/response envelopes over the instance messenger.

An instance leader serves operator and peer requests on its messenger,
grouped in modules that a client can list before it calls them:

core      ``kvbm.leader.control.describe_instance`` -> identity, block size,
          parallelism, tier capacities, per-worker layouts, role, config,
          host and start time.
dev       ``kvbm.connector.leader.reset`` {tiers?} -> drop every inactive
          (cached, unreferenced) block of the named tiers (G2, G3). An
          explicit list naming a tier this leader lacks fails before any tier
          is reset; without a list every configured tier is reset and the
          rest are reported as skipped.
metrics   ``kvbm.leader.control.metrics.snapshot`` -> per-pool occupancy and
          counters, transfer sessions in flight, conditional-disaggregation
          counters.
transfer  ``kvbm.leader.control.open_session`` / ``pull_from_session`` /
          ``close_session`` / ``search_prefix``: the remote-search session
          handlers under their control-plane names.

Replies are ``{"ok": true, "value": ...}`` or ``{"ok": false, "error":
{"kind", "message"}}``; :class:`LeaderControlClient` turns the latter into
:class:`ControlError`.

Parity: crates/kvbm-protocols/src/control/{mod.rs:73-210 (ModuleId,
list_modules, ControlError, ControlReply), modules/core.rs (describe
instance), modules/dev.rs:41-125 (ResetRequest / ResetResponse /
plan_reset), modules/metrics.rs (snapshot), modules/transfer.rs (session
handler names), client.rs (LeaderControlClient)}.
"""

from __future__ import annotations

import os
import socket
import time
from typing import Any, Callable

LIST_MODULES = "kvbm.leader.control.list_modules"
DESCRIBE_INSTANCE = "kvbm.leader.control.describe_instance"
RESET = "kvbm.connector.leader.reset"
METRICS_SNAPSHOT = "kvbm.leader.control.metrics.snapshot"
OPEN_SESSION = "kvbm.leader.control.open_session"
PULL_FROM_SESSION = "kvbm.leader.control.pull_from_session"
CLOSE_SESSION = "kvbm.leader.control.close_session"
SEARCH_PREFIX = "kvbm.leader.control.search_prefix"

RESET_TIERS = ("g2", "g3")  # resettable tiers, in reset order


class ControlError(RuntimeError):
    def __init__(self, kind: str, message: str):
        super().__init__(f"{kind}: {message}")
        self.kind, self.message = kind, message


def plan_reset(tiers: list[str] | None, available: set[str]) -> tuple[list[str], list[str]]:
    """(tiers to reset, tiers skipped as unconfigured). An explicit list must name configured tiers
    only (checked for all of them before anything is reset); duplicates are dropped."""
    if tiers is not None:
        for t in tiers:
            if t not in RESET_TIERS:
                raise ControlError("unknown_tier", f"tier {t!r} (resettable: {', '.join(RESET_TIERS)})")
            if t not in available:
                raise ControlError("tier_not_configured", f"tier {t!r} is not configured on this leader")
        out = []
        for t in tiers:
            if t not in out:
                out.append(t)
        return out, []
    return [t for t in RESET_TIERS if t in available], [t for t in RESET_TIERS if t not in available]


def _layout_description(tier: str, layout) -> dict:
    c = layout.config
    return {"tier": tier, "layout_type": getattr(layout, "kind", "?"),
            "block_layout": getattr(getattr(layout, "block_layout", None), "value", "?"),
            "location": getattr(layout, "location", "?"),
            "config": {"num_blocks": c.num_blocks, "num_layers": c.num_layers, "outer_dim": c.outer_dim,
                       "page_size": c.page_size, "num_heads": c.num_heads, "head_dim": c.head_dim,
                       "dtype": str(c.torch_dtype).replace("torch.", "")}}


def _pool(tier: str, mgr) -> dict:
    m = dict(mgr.metrics())
    return {"tier": tier, "total_blocks": mgr.total_blocks(), "available_blocks": mgr.available_blocks(),
            "inactive_blocks": mgr.inactive_len(), "active_blocks": mgr.active_len(),
            "reset_blocks": mgr.reset_len(), **m}


class LeaderControl:
    """Serves the control modules of one instance leader on ``messenger``.

    ``worker_layouts`` lists each worker's ``{tier: KvLayout}``; ``holder`` / ``search`` are the
    instance's remote-search holder and initiator (the transfer module is offered when both
    exist); ``role``, ``config``, ``parallelism`` and ``cd_stats`` feed describe / metrics."""

    def __init__(self, leader, messenger, block_size: int | None = None, worker_layouts: list[dict] | None = None,
                 holder=None, search=None, role: str | None = None, config: dict | None = None,
                 parallelism: dict | None = None, cd_stats: Callable[[], dict] | None = None,
                 hub_instance_id: str | None = None):
        self.leader, self.messenger = leader, messenger
        self.block_size = block_size
        self.worker_layouts = list(worker_layouts or [])
        self.holder, self.search = holder, search
        self.role, self.config, self.parallelism = role, config, parallelism
        self.cd_stats = cd_stats
        self.hub_instance_id = hub_instance_id
        self.started_at = time.time()
        self.modules = ["core", "dev", "metrics"] + (["transfer"] if holder is not None and search is not None
                                                     else [])
        self._serve(LIST_MODULES, lambda req: {"modules": list(self.modules)})
        self._serve(DESCRIBE_INSTANCE, self.describe)
        self._serve(RESET, self.reset)
        self._serve(METRICS_SNAPSHOT, self.metrics_snapshot)
        if "transfer" in self.modules:
            self._serve(OPEN_SESSION, holder._open)
            self._serve(CLOSE_SESSION, holder._close)
            self._serve(PULL_FROM_SESSION, search._pull_rpc)
            self._serve(SEARCH_PREFIX, self._search_prefix)

    def _serve(self, name: str, fn: Callable[[Any], Any]) -> None:
        def wrapped(req):
            try:
                return {"ok": True, "value": fn(req or {})}
            except ControlError as e:
                return {"ok": False, "error": {"kind": e.kind, "message": e.message}}
            except Exception as e:  # noqa: BLE001 - reported to the caller, not raised in the server loop
                return {"ok": False, "error": {"kind": type(e).__name__, "message": str(e)}}
        self.messenger.register_handler(name, wrapped)

    # ------------------------------------------------------------- modules
    def _tiers(self) -> dict[str, object]:
        t = {"g2": self.leader.g2}
        if getattr(self.leader, "g3", None) is not None:
            t["g3"] = self.leader.g3
        return t

    def describe(self, req: dict | None = None) -> dict:
        tiers = self._tiers()
        return {
            "instance_id": str(self.leader.instance_id),
            "hub_instance_id": self.hub_instance_id,
            "worker_ids": list(range(len(self.worker_layouts))),
            "block_size": self.block_size,
            "parallelism": self.parallelism,
            "tier_capacity": [{"tier": k, "total_blocks": m.total_blocks()} for k, m in tiers.items()],
            "workers": [{"worker_id": i, "layouts": [_layout_description(t, l) for t, l in wl.items()]}
                        for i, wl in enumerate(self.worker_layouts)],
            "modules": list(self.modules),
            "role": self.role,
            "config": self.config,
            "host": {"hostname": socket.gethostname(), "pid": os.getpid()},
            "started_at": self.started_at,
        }

    def reset(self, req: dict) -> dict:
        tiers = self._tiers()
        todo, skipped = plan_reset(req.get("tiers"), set(tiers))
        done, failed = [], []
        for t in todo:
            try:
                tiers[t].reset_inactive_pool()
                done.append(t)
            except Exception as e:  # noqa: BLE001 - blocks still in use: reported per tier
                failed.append({"tier": t, "message": str(e)})
        out = {"reset": done, "failed": failed}
        if skipped:
            out["skipped_unconfigured"] = skipped
        return out

    def metrics_snapshot(self, req: dict | None = None) -> dict:
        sessions = self.holder.open_sessions() if self.holder is not None else 0
        return {"gathered_at_unix_ms": int(time.time() * 1000), "sessions_inflight": sessions,
                "pools": [_pool(k, m) for k, m in self._tiers().items()],
                "cd": dict(self.cd_stats()) if self.cd_stats is not None else None}

    def _search_prefix(self, req: dict) -> dict:
        hashes = [int(h) for h in req["hashes"]]
        found = self.search.search(hashes)
        local = self.leader.g2.count_prefix(hashes)
        return {"local_g2_blocks": local,
                "remote": None if found is None else {"holder": found[0], "blocks": found[1]}}


class LeaderControlClient:
    """Typed calls to a leader's control plane at messenger ``address``."""

    def __init__(self, messenger, address, timeout: float = 10.0):
        self.m, self.addr, self.timeout = messenger, address, timeout

    def _call(self, handler: str, payload: dict | None = None):
        from ..runtime.messenger import RpcError

        try:
            r = self.m.call(self.addr, handler, payload or {}, timeout=self.timeout)
        except RpcError as e:
            if "no handler" in str(e):
                raise ControlError("module_not_offered", f"{handler} is not served by this leader") from e
            raise
        if not r.get("ok"):
            e = r.get("error", {})
            raise ControlError(e.get("kind", "error"), e.get("message", ""))
        return r["value"]

    def list_modules(self) -> list[str]:
        return self._call(LIST_MODULES)["modules"]

    def describe(self) -> dict:
        return self._call(DESCRIBE_INSTANCE)

    def reset(self, tiers: list[str] | None = None) -> dict:
        return self._call(RESET, {"tiers": tiers} if tiers is not None else {})

    def metrics(self) -> dict:
        return self._call(METRICS_SNAPSHOT)

    def open_session(self, hashes: list[int], initiator: int = 0) -> dict:
        return self._call(OPEN_SESSION, {"initiator": str(initiator), "hashes": [str(h) for h in hashes]})

    def pull_from_session(self, holder: int, session: dict, hashes: list[int]) -> dict:
        return self._call(PULL_FROM_SESSION, {"holder": holder, "session": session, "hashes": [str(h) for h in hashes]})

    def close_session(self, sid: str) -> dict:
        return self._call(CLOSE_SESSION, {"sid": sid})

    def search_prefix(self, hashes: list[int]) -> dict:
        return self._call(SEARCH_PREFIX, {"hashes": [str(h) for h in hashes]})
