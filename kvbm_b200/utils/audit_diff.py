"""Offline equivalence check of two ``kvbm_audit`` traces.

Reads two log files, keeps the audit records (JSON objects written by
``utils.tracing.audit``, one per line, optionally after a logging prefix;
``key=value`` records after a ``kvbm_audit:`` tag are accepted too), and
compares their ``(event, role, request_id)`` signature sequences. Exit code
0 when equivalent, 1 on divergence (a per-position left/right diff is
printed), 2 on usage errors.

    python -m kvbm_b200.utils.audit_diff LEFT.log RIGHT.log \
        [--filter-prefixes gnmt_,transfer_] [--multiset] [--normalize-request-ids]

* ``--multiset``: equal when every signature occurs equally often, in any order.
* ``--normalize-request-ids``: rename request ids to ``req-1, req-2, ...`` in
  order of first appearance per file (two live runs get different ids).
* ``--filter-prefixes``: drop events whose name starts with any prefix.

Parity: crates/kvbm-connector/src/bin/audit_diff.rs.
"""

from __future__ import annotations

import argparse
import json
import re
import shlex
import sys
from collections import Counter

Signature = tuple[str, str | None, str | None]
_KV_TAG = "kvbm_audit:"


def parse_line(line: str) -> dict | None:
    """One audit record from a log line, or None."""
    i = line.find("{")
    if i >= 0 and '"event"' in line:
        try:
            d = json.loads(line[i:])
            if isinstance(d, dict) and "event" in d:
                return d
        except ValueError:
            pass
    j = line.find(_KV_TAG)
    if j >= 0:
        out = {}
        try:
            parts = shlex.split(line[j + len(_KV_TAG):])
        except ValueError:
            return None
        for p in parts:
            if "=" in p:
                k, v = p.split("=", 1)
                out[k] = v
        return out if "event" in out else None
    return None


def signatures(lines, filter_prefixes=(), normalize=False) -> list[Signature]:
    ids: dict[str, str] = {}
    out = []
    for line in lines:
        d = parse_line(line)
        if d is None:
            continue
        ev = str(d["event"])
        if any(ev.startswith(p) for p in filter_prefixes):
            continue
        rid = d.get("request_id", d.get("request"))
        rid = None if rid is None else str(rid)
        if normalize and rid is not None:
            rid = ids.setdefault(rid, f"req-{len(ids) + 1}")
        role = d.get("role")
        out.append((ev, None if role is None else str(role), rid))
    return out


def compare(left: list[Signature], right: list[Signature], multiset: bool = False) -> list[str]:
    """Differences as printable lines (empty when equivalent)."""
    if multiset:
        cl, cr = Counter(left), Counter(right)
        diff = []
        for sig in sorted(set(cl) | set(cr), key=lambda s: tuple("" if x is None else x for x in s)):
            if cl[sig] != cr[sig]:
                diff.append(f"{sig}: left x{cl[sig]}, right x{cr[sig]}")
        return diff
    diff = []
    for k in range(max(len(left), len(right))):
        a = left[k] if k < len(left) else None
        b = right[k] if k < len(right) else None
        if a != b:
            diff.append(f"[{k}] L={a} R={b}")
    return diff


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("left")
    p.add_argument("right")
    p.add_argument("--filter-prefixes", default="")
    p.add_argument("--multiset", action="store_true")
    p.add_argument("--normalize-request-ids", action="store_true")
    p.add_argument("--max-lines", type=int, default=50)
    try:
        a = p.parse_args(argv)
    except SystemExit:
        return 2
    prefixes = tuple(x for x in re.split(r"[,\s]+", a.filter_prefixes) if x)
    try:
        with open(a.left) as fl, open(a.right) as fr:
            left = signatures(fl, prefixes, a.normalize_request_ids)
            right = signatures(fr, prefixes, a.normalize_request_ids)
    except OSError as e:
        print(f"audit_diff: {e}", file=sys.stderr)
        return 2
    diff = compare(left, right, a.multiset)
    if not diff:
        print(f"equivalent: {len(left)} audit events")
        return 0
    print(f"divergent: {len(diff)} difference(s) ({len(left)} vs {len(right)} events)")
    for line in diff[: a.max_lines]:
        print("  " + line)
    return 1


if __name__ == "__main__":
    sys.exit(main())
