"""``kvbmctl``: command-line view of a running hub.

    python -m kvbm_b200.hub.kvbmctl --hub http://127.0.0.1:1337 instances
    python -m kvbm_b200.hub.kvbmctl --hub ... query <hash> [<hash> ...]
    python -m kvbm_b200.hub.kvbmctl --hub ... router

Parity: crates/kvbm-hub/src/bin/kvbmctl.rs and render.rs (table rendering).
"""

from __future__ import annotations

import argparse
import json
import sys

from .client import HubClient


def render_table(rows: list[dict], cols: list[str]) -> str:
    widths = {c: max([len(c)] + [len(str(r.get(c, ""))) for r in rows]) for c in cols}
    line = "  ".join(c.upper().ljust(widths[c]) for c in cols)
    out = [line]
    for r in rows:
        out.append("  ".join(str(r.get(c, "")).ljust(widths[c]) for c in cols))
    return "\n".join(out)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="kvbmctl")
    p.add_argument("--hub", default="http://127.0.0.1:1337")
    p.add_argument("--json", action="store_true")
    sub = p.add_subparsers(dest="cmd", required=True)
    sub.add_parser("health")
    sub.add_parser("config")
    i = sub.add_parser("instances")
    i.add_argument("--role", default=None)
    q = sub.add_parser("query")
    q.add_argument("hashes", nargs="+")
    sub.add_parser("router")
    a = p.parse_args(argv)
    c = HubClient(a.hub)
    if a.cmd == "health":
        out = c.health()
    elif a.cmd == "config":
        out = c.config()
    elif a.cmd == "instances":
        rows = c.instances(a.role)
        if not a.json:
            print(render_table([dict(r, features=",".join(r["features"])) for r in rows],
                               ["instance_id", "role", "features", "address"]))
            return 0
        out = rows
    elif a.cmd == "query":
        out = c.query([int(h, 0) for h in a.hashes])
    else:
        out = {"targets": c.targets(), **c.router_counters()}
    print(json.dumps(out, indent=None if a.json else 2, default=str))
    return 0


if __name__ == "__main__":
    sys.exit(main())
