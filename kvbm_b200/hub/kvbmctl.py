"""``kvbmctl``: operator tool for a running hub.

    kvbmctl --hub URL health | instances [--role R] | query <hash>... | router
    kvbmctl --hub URL config                       # the hub's aggregate configuration
    kvbmctl --hub URL config vllm [--features indexer,disagg] [--role prefill|decode]
                                  [--kvbm a.b=value ...] [--kvbm-config JSON]
        -> --block-size N --max-model-len M --kv-transfer-config '<json>'
    kvbmctl --hub URL p2p pin   --instance-id H --hashes h1,h2,...
    kvbmctl --hub URL p2p pull  --from H --to P --session JSON [--hashes ...]
    kvbmctl --hub URL p2p unpin --instance-id H --session SID
    kvbmctl --hub URL p2p xfer  --from H --to P --hashes h1,h2,...
    kvbmctl --hub URL control --instance-id I modules | describe | metrics | reset [--tiers g2,g3]

``config vllm`` renders the vLLM flags that connect an engine to this hub:
the hub's block size and maximum sequence length, and a
``--kv-transfer-config`` whose ``kv_connector_extra_config`` selects the
features (validated against the hub's enabled set; ``disagg`` pulls in
``p2p``; the prefill router only for a prefill role unless asked for), the
conditional-disaggregation role, and the operator's overrides. Overrides are
applied lowest to highest: the hub's base configuration, ``--kvbm-config``,
each ``--kvbm path=value``; the hub-owned fields (hub URL and features,
disaggregation role) are applied last and always win. The result is checked
by loading it as a block-manager configuration.

``control`` calls an instance leader's control plane (its messenger
address comes from the hub): the modules it serves, its description, a
metrics snapshot, or a reset of its cached (inactive) G2/G3 blocks.

``p2p`` drives the remote-search transfer sessions by hand: ``pin`` opens a
session on a holder (its blocks stay pinned), ``pull`` makes another
instance copy a pinned session's blocks into its G2, ``unpin`` closes the
session, ``xfer`` does all three.

Parity: crates/kvbm-hub/src/bin/kvbmctl.rs, render.rs:82-300
(resolve_features, render_vllm_cli, shell quoting), features/p2p/cli.rs
(pin / pull / unpin / xfer), kvbm-protocols/src/control/client.rs (the
leader control client).
"""

from __future__ import annotations

import argparse
import copy
import json
import os
import sys

from .client import HubClient

SELECTABLE = ("indexer", "p2p", "disagg", "prefill_router")
DEPENDENCIES = {"disagg": ("p2p",)}


def render_table(rows: list[dict], cols: list[str]) -> str:
    widths = {c: max([len(c)] + [len(str(r.get(c, ""))) for r in rows]) for c in cols}
    line = "  ".join(c.upper().ljust(widths[c]) for c in cols)
    out = [line]
    for r in rows:
        out.append("  ".join(str(r.get(c, "")).ljust(widths[c]) for c in cols))
    return "\n".join(out)


# ------------------------------------------------------------- config vllm
def resolve_features(hub_features: list[str], requested: list[str]) -> list[str]:
    enabled = [f for f in SELECTABLE if f in hub_features]
    if not requested:
        sel = list(enabled)
    else:
        sel = []
        for f in requested:
            if f not in SELECTABLE:
                raise ValueError(f"unknown feature {f!r}; valid features: {', '.join(SELECTABLE)}")
            if f not in enabled:
                raise ValueError(f"feature {f!r} is not enabled on the hub (enabled: {', '.join(enabled) or '<none>'})")
            if f not in sel:
                sel.append(f)
    for f in list(sel):  # dependency closure
        for d in DEPENDENCIES.get(f, ()):
            if d not in enabled:
                raise ValueError(f"feature {f!r} needs {d!r}, which the hub does not enable")
            if d not in sel:
                sel.append(d)
    if "disagg" in sel and "prefill_router" in enabled and "prefill_router" not in sel:
        sel.append("prefill_router")
    return [f for f in SELECTABLE if f in sel]


def _deep_merge(dst: dict, src: dict) -> dict:
    for k, v in src.items():
        if isinstance(v, dict) and isinstance(dst.get(k), dict):
            _deep_merge(dst[k], v)
        else:
            dst[k] = copy.deepcopy(v)
    return dst


def _parse_value(v: str):
    try:
        return json.loads(v)
    except ValueError:
        return v


def apply_overrides(extra: dict, config_json: str | None, overrides: list[str]) -> dict:
    if config_json:
        blob = json.loads(config_json)
        if not isinstance(blob, dict):
            raise ValueError("--kvbm-config must be a JSON object")
        _deep_merge(extra, blob)
    for o in overrides:
        if "=" not in o:
            raise ValueError(f"--kvbm expects KEY.PATH=VALUE, got {o!r}")
        path, val = o.split("=", 1)
        keys = path.split(".")
        cur = extra
        for k in keys[:-1]:
            cur = cur.setdefault(k, {})
            if not isinstance(cur, dict):
                raise ValueError(f"--kvbm {path}: {k!r} is not a table")
        cur[keys[-1]] = _parse_value(val)
    return extra


def shell_single_quote(s: str) -> str:
    return "'" + s.replace("'", "'\\''") + "'"


def render_vllm_cli(hub_cfg: dict, hub_url: str, features: list[str] | None = None, role: str | None = None,
                    overrides: list[str] = (), config_json: str | None = None,
                    kv_connector: str = "KvbmConnector", kv_role: str = "kv_both",
                    kv_load_failure_policy: str = "recompute",
                    kv_connector_module_path: str = "kvbm_b200.connector.vllm_connector") -> str:
    from ..utils.config import KvbmConfig

    eff = resolve_features(list(hub_cfg.get("features", [])), list(features or []))
    if role != "prefill" and "prefill_router" not in (features or []):
        eff = [f for f in eff if f != "prefill_router"]
    if "disagg" in eff and role not in ("prefill", "decode"):
        raise ValueError("the disagg feature needs --role prefill or --role decode")
    if "disagg" not in eff and role is not None:
        raise ValueError("--role applies only with the disagg feature")
    extra: dict = {}
    if hub_cfg.get("base_config"):
        _deep_merge(extra, hub_cfg["base_config"])
    apply_overrides(extra, config_json, list(overrides))
    authoritative = {"hub": {"url": hub_url, "features": eff}}
    if "disagg" in eff:
        authoritative["disagg"] = {"role": role}
    _deep_merge(extra, authoritative)
    KvbmConfig.load(extra, env={}, system_toml=None)  # rejects unknown keys and bad values
    ktc = {"kv_connector": kv_connector, "kv_role": kv_role, "kv_load_failure_policy": kv_load_failure_policy,
           "kv_connector_module_path": kv_connector_module_path, "kv_connector_extra_config": extra}
    parts = []
    if hub_cfg.get("block_size"):
        parts.append(f"--block-size {hub_cfg['block_size']}")
    if hub_cfg.get("max_seq_len"):
        parts.append(f"--max-model-len {hub_cfg['max_seq_len']}")
    parts.append("--kv-transfer-config " + shell_single_quote(json.dumps(ktc, separators=(",", ":"))))
    return " ".join(parts)


# --------------------------------------------------------------------- p2p
def _hashes(s: str | None) -> list[str]:
    return [str(int(h, 0)) for h in s.split(",") if h] if s else []


def run_p2p(a, client: HubClient) -> dict:
    from ..engine.remote_search import CLOSE, OPEN, PULL
    from ..runtime.messenger import Messenger

    m = Messenger(instance_id=0)
    try:
        if a.p2p == "pin":
            addr = client.peer(a.instance_id)["address"]
            return m.call(addr, OPEN, {"initiator": "0", "hashes": _hashes(a.hashes)}, timeout=a.timeout)
        if a.p2p == "unpin":
            addr = client.peer(a.instance_id)["address"]
            return m.call(addr, CLOSE, {"sid": a.session}, timeout=a.timeout)
        to = client.peer(getattr(a, "to"))["address"]
        if a.p2p == "pull":
            session = json.loads(a.session)
            hashes = _hashes(a.hashes) or [str(h) for h in session.get("hashes", [])]
            return m.call(to, PULL, {"holder": getattr(a, "from"), "hashes": hashes, "session": session},
                          timeout=a.timeout)
        return m.call(to, PULL, {"holder": getattr(a, "from"), "hashes": _hashes(a.hashes)}, timeout=a.timeout)
    finally:
        m.close()


def run_control(a, client: HubClient):
    from ..engine.control import LeaderControlClient
    from ..runtime.messenger import Messenger

    m = Messenger(instance_id=0)
    try:
        ctl = LeaderControlClient(m, client.peer(a.instance_id)["address"], timeout=a.timeout)
        if a.action == "modules":
            return {"modules": ctl.list_modules()}
        if a.action == "describe":
            return ctl.describe()
        if a.action == "metrics":
            return ctl.metrics()
        return ctl.reset([t for t in a.tiers.split(",") if t] if a.tiers else None)
    finally:
        m.close()


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="kvbmctl")
    p.add_argument("--hub", default=os.environ.get("KVBMCTL_HUB", "http://127.0.0.1:1337"),
                   help="hub URL (default: $KVBMCTL_HUB, else http://127.0.0.1:1337)")
    p.add_argument("--json", action="store_true")
    sub = p.add_subparsers(dest="cmd", required=True)
    sub.add_parser("health")
    c = sub.add_parser("config")
    csub = c.add_subparsers(dest="target")
    v = csub.add_parser("vllm")
    v.add_argument("--features", default="")
    v.add_argument("--role", default=None)
    v.add_argument("--kvbm", action="append", default=[])
    v.add_argument("--kvbm-config", default=None)
    v.add_argument("--kv-connector", default="KvbmConnector")
    v.add_argument("--kv-role", default="kv_both")
    v.add_argument("--kv-load-failure-policy", default="recompute")
    v.add_argument("--kv-connector-module-path", default="kvbm_b200.connector.vllm_connector")
    i = sub.add_parser("instances")
    i.add_argument("--role", default=None)
    q = sub.add_parser("query")
    q.add_argument("hashes", nargs="+")
    sub.add_parser("router")
    pp = sub.add_parser("p2p")
    psub = pp.add_subparsers(dest="p2p", required=True)
    for name in ("pin", "pull", "unpin", "xfer"):
        s = psub.add_parser(name)
        s.add_argument("--timeout", type=float, default=30.0)
        if name in ("pin", "unpin"):
            s.add_argument("--instance-id", type=int, required=True)
        else:
            s.add_argument("--from", type=int, required=True)
            s.add_argument("--to", type=int, required=True)
        if name in ("pull", "unpin"):
            s.add_argument("--session", required=True, help="unpin: the session id; pull: pin's JSON output")
        s.add_argument("--hashes", default=None, required=name in ("pin", "xfer"))
    ct = sub.add_parser("control")
    ct.add_argument("--instance-id", type=int, required=True)
    ct.add_argument("--timeout", type=float, default=10.0)
    ct.add_argument("action", choices=["modules", "describe", "metrics", "reset"])
    ct.add_argument("--tiers", default=None, help="reset: comma list of g2,g3 (default: every configured tier)")
    ix = sub.add_parser("indexer", help="query the hub's KV block index")
    ixs = ix.add_subparsers(dest="ix", required=True)
    ixs.add_parser("config")
    ixs.add_parser("get-instances", help="instances registered to the indexer (not all of them emit events)")
    bp = ixs.add_parser("by-pos", help="indexed blocks at a position bucket")
    bp.add_argument("pos", type=int)
    iq = ixs.add_parser("query", help="which instances hold a block hash (decimal or 0x, e.g. a by-pos hash_u128)")
    iq.add_argument("hash")
    dg = sub.add_parser("disagg", help="the hub's conditional-disaggregation registry")
    dgs = dg.add_subparsers(dest="dg", required=True)
    dgs.add_parser("instances", help="registered prefill / decode instances and the queue depth")
    cal = sub.add_parser("calibrate", help="run a prefill worker's calibration sweep through the hub")
    cal.add_argument("--instance-id", type=int, required=True)
    cal.add_argument("--seq", default=None, help="comma list of input lengths (default: the engine's ladder)")
    cal.add_argument("--osl", type=int, default=None)
    cal.add_argument("--seed", type=int, default=None)
    cal.add_argument("--max-isl-fraction", type=float, default=None)
    cal.add_argument("--no-warmup", action="store_true")
    cal.add_argument("--force", action="store_true", help="re-run even when the worker has a cached result")
    cal.add_argument("--timeout", type=float, default=1800.0)
    a = p.parse_args(argv)
    client = HubClient(a.hub)
    if a.cmd == "health":
        out = client.health()
    elif a.cmd == "config" and a.target == "vllm":
        try:
            print(render_vllm_cli(client.config(), a.hub, [f for f in a.features.split(",") if f], a.role,
                                  a.kvbm, a.kvbm_config, a.kv_connector, a.kv_role, a.kv_load_failure_policy,
                                  a.kv_connector_module_path))
        except ValueError as e:
            print(f"kvbmctl: {e}", file=sys.stderr)
            return 2
        return 0
    elif a.cmd == "config":
        out = client.config()
    elif a.cmd == "instances":
        rows = client.instances(a.role)
        if not a.json:
            print(render_table([dict(r, features=",".join(r["features"])) for r in rows],
                               ["instance_id", "role", "features", "address"]))
            return 0
        out = rows
    elif a.cmd == "query":
        out = client.query([int(h, 0) for h in a.hashes])
    elif a.cmd == "control":
        from ..engine.control import ControlError

        try:
            out = run_control(a, client)
        except ControlError as e:
            print(f"kvbmctl: {e}", file=sys.stderr)
            return 2
    elif a.cmd == "indexer":
        if a.ix == "config":
            out = client.index_config()
        elif a.ix == "get-instances":
            out = {"instances": client.index_instances()}
        elif a.ix == "by-pos":
            out = client.index_by_position(a.pos)
        else:
            out = client.query([int(a.hash, 0)])
    elif a.cmd == "disagg":
        out = client.disagg_instances()
    elif a.cmd == "calibrate":
        req = {k: v for k, v in {"seq": [int(x) for x in a.seq.split(",")] if a.seq else None, "osl": a.osl,
                                  "seed": a.seed, "max_isl_fraction": a.max_isl_fraction,
                                  "warmup": False if a.no_warmup else None}.items() if v is not None}
        try:
            res = client.run_calibration(a.instance_id, req, force=a.force, timeout=a.timeout)
        except RuntimeError as e:
            print(f"kvbmctl: {e}", file=sys.stderr)
            return 2
        if a.json:
            out = res
        else:
            pm = res["results"]["performance_model"]
            print(f"instance {a.instance_id}: {'cached' if res['from_cache'] else 'measured'} over "
                  f"ISL {res['resolved']['seq']}, OSL {res['resolved']['osl']}")
            print(f"  TTFT(us) = {pm['t2ft_intercept']:.1f} + {pm['t2ft_linear']:.4g}*ISL + "
                  f"{pm['t2ft_quadratic']:.4g}*ISL^2   (R^2 {pm['t2ft_fit_r2']:.4f})")
            print(f"  ITL(us)  = {pm['t2tl_intercept']:.1f} + {pm['t2tl_slope']:.4g}*position   "
                  f"(R^2 {pm['t2tl_fit_r2']:.4f})")
            print(f"  n_opt {res['results']['n_opt']}  n_att {res['results']['n_att']}")
            for c_ in res["resolved"].get("clamps", []):
                print(f"  clamp: {c_}")
            return 0
    elif a.cmd == "p2p":
        out = run_p2p(a, client)
        if a.p2p == "pin" and out.get("sid") is not None:
            out = dict(out, hashes=_hashes(a.hashes))
    else:
        out = {"targets": client.targets(), **client.router_counters()}
    print(json.dumps(out, indent=None if a.json else 2, default=str))
    return 0


if __name__ == "__main__":
    sys.exit(main())
