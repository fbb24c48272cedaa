"""CPU-only block-pool plumbing benchmark (no GPU; G2-only host pool).

Workload: ``requests`` synthetic requests, token ids uniform in [0, 32000),
lengths uniform in [512, 4096]; half of them start with one of 8 fixed
1,024-token prefixes. For each request: hash its complete 16-token blocks,
match the cached prefix, allocate the rest (evicting under pressure),
register them, release everything. Reports the block hit rate, requests/s
and blocks/s through the framework's block handles (``BlockManager``) and
through the native pool's batch calls (``native_batch``), and checks the
KV-event log (Create /
Remove per sequence hash, in order) against an independent pure-Python model
of the same pool semantics (LRU eviction) - the "event-log equality" check.

    python -m kvbm_b200.bench.pool_bench --blocks 65536 --requests 4096
    python -m kvbm_b200.bench.pool_bench --micro     # per-block match (active / inactive) and drop

Parity: benches/block_manager.rs (match active hit, inactive hit, bulk drop).
"""

from __future__ import annotations

import argparse
import collections
import json
import time

import numpy as np

from .. import _core_native as core
from ..logical.manager import BlockManager, Tier
from ..logical.sequence import sequence_hashes


def make_workload(n: int, seed: int = 0, vocab: int = 32000, block: int = 16):
    rng = np.random.default_rng(seed)
    prefixes = [rng.integers(0, vocab, 1024, dtype=np.int32) for _ in range(8)]
    reqs = []
    for i in range(n):
        length = int(rng.integers(512, 4097))
        toks = rng.integers(0, vocab, length, dtype=np.int32)
        if rng.random() < 0.5:
            p = prefixes[int(rng.integers(0, 8))]
            k = min(1024, length)
            toks[:k] = p[:k]
        reqs.append(toks)
    return [sequence_hashes(t, block) for t in reqs]


class PyLruPool:
    """Independent model: reset FIFO, LRU inactive, Create on first presence, Remove on eviction."""

    def __init__(self, n: int):
        self.free = collections.deque(range(n))
        self.inactive: collections.OrderedDict[int, int] = collections.OrderedDict()
        self.events: list[tuple[str, int]] = []

    def process(self, hashes: list[int]) -> int:
        hit = 0
        for h in hashes:
            if h in self.inactive:
                hit += 1
            else:
                break
        matched = hashes[:hit]
        held = {h: self.inactive.pop(h) for h in matched}
        need = hashes[hit:]
        if len(self.free) + len(self.inactive) < len(need):
            for h, b in held.items():  # release matched blocks back in order
                self.inactive[h] = b
            return -1
        blocks = []
        for _ in need:
            if self.free:
                blocks.append(self.free.popleft())
            else:
                h, b = self.inactive.popitem(last=False)
                self.events.append(("remove", h))
                blocks.append(b)
        for h in need:
            self.events.append(("create", h))
        # release: matched (in order) then new blocks (in order) become inactive
        for h in matched:
            self.inactive[h] = held[h]
        for h, b in zip(need, blocks):
            self.inactive[h] = b
        return hit


def run_native(workload, blocks: int, backend: str = "lru"):
    q = core.EventQueue(all_events=True)
    mgr = BlockManager(blocks, 16, backend, Tier.G2, registry=core.Registry(events=q))
    hits = total = 0
    log = []
    t0 = time.perf_counter()
    for hashes in workload:
        matched = mgr.match_blocks(hashes)
        need = hashes[len(matched):]
        got = mgr.allocate_blocks(len(need))
        if got is None:
            for b in matched:
                b.release()
            continue
        imm = mgr.register_mutable(got, need)
        for b in matched:
            b.release()
        for b in imm:
            b.release()
        hits += len(matched)
        total += len(hashes)
        log.extend(q.drain())
    dt = time.perf_counter() - t0
    return {"hit_rate": hits / max(1, total), "seconds": dt, "blocks": total, "events": log}


def run_batch(workload, blocks: int, backend: str = "lru"):
    """The same request loop on the native pool's batch calls (block ids, no Python block handles)."""
    q = core.EventQueue(all_events=True)
    pool = core.BlockPool(blocks, 16, backend, int(Tier.G2), core.Registry(events=q), "allow")
    hits = total = 0
    log = []
    t0 = time.perf_counter()
    for hashes in workload:
        matched = pool.match_prefix(hashes)
        need = hashes[len(matched):]
        got = pool.allocate(len(need))
        if got is None:
            pool.release_many(matched)
            continue
        ids, _evicted = got
        reg = pool.stage_and_register(ids, need)
        pool.release_many(matched)
        pool.release_many([bid for bid, _ in reg])
        hits += len(matched)
        total += len(hashes)
        log.extend(q.drain())
    dt = time.perf_counter() - t0
    return {"hit_rate": hits / max(1, total), "seconds": dt, "blocks": total, "events": log}


def micro(n: int = 4096, reps: int = 20, backend: str = "lru") -> dict:
    """Per-block cost of the pool's three hot calls, as the reference's block-manager
    micro-benchmarks time them: a prefix match that hits blocks still held by another
    request (active), one that hits released blocks (inactive: reactivated from the
    eviction index), and dropping a batch of registered blocks. Native batch calls and
    Python block handles, ns per block (median of ``reps``)."""
    hashes = sequence_hashes(list(range(n * 16)), 16)
    out = {}

    def med(xs):
        return round(sorted(xs)[len(xs) // 2] * 1e9 / n, 1)

    # native batch API
    pool = core.BlockPool(n + 8, 16, backend, int(Tier.G2), core.Registry(), "allow")
    ids, _ = pool.allocate(n)
    held = [bid for bid, _ in pool.stage_and_register(ids, hashes)]
    t_act, t_inact, t_drop = [], [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        m = pool.match_prefix(hashes)
        t_act.append(time.perf_counter() - t0)
        pool.release_many(m)
    pool.release_many(held)  # every block inactive now
    for _ in range(reps):
        t0 = time.perf_counter()
        m = pool.match_prefix(hashes)
        t_inact.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        pool.release_many(m)
        t_drop.append(time.perf_counter() - t0)
    out["native_batch_ns_per_block"] = {"match_active": med(t_act), "match_inactive": med(t_inact),
                                        "drop": med(t_drop)}
    # Python block handles
    mgr = BlockManager(n + 8, 16, inactive=backend, tier=Tier.G2)
    got = mgr.allocate_blocks(n)
    owner = mgr.register_mutable(got, hashes)
    t_act, t_inact, t_drop = [], [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        m = mgr.match_blocks(hashes)
        t_act.append(time.perf_counter() - t0)
        for b in m:
            b.release()
    for b in owner:
        b.release()
    for _ in range(reps):
        t0 = time.perf_counter()
        m = mgr.match_blocks(hashes)
        t_inact.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        for b in m:
            b.release()
        t_drop.append(time.perf_counter() - t0)
    out["handles_ns_per_block"] = {"match_active": med(t_act), "match_inactive": med(t_inact), "drop": med(t_drop)}
    out["blocks"] = n
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--blocks", type=int, default=65536)
    p.add_argument("--requests", type=int, default=4096)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--backend", default="lru")
    p.add_argument("--check", action="store_true", default=True)
    p.add_argument("--micro", action="store_true", help="only the per-block match / drop micro-benchmarks")
    a = p.parse_args(argv)
    if a.micro:
        out = micro(backend=a.backend)
        print(json.dumps(out))
        return out
    wl = make_workload(a.requests, a.seed)
    nat = run_native(wl, a.blocks, a.backend)
    out = {"requests": a.requests, "blocks": a.blocks, "backend": a.backend,
           "hit_rate": round(nat["hit_rate"], 4), "requests_per_s": round(a.requests / nat["seconds"], 1),
           "blocks_per_s": round(nat["blocks"] / nat["seconds"], 1), "events": len(nat["events"])}
    if a.check and a.backend == "lru":
        model = PyLruPool(a.blocks)
        hits = sum(max(0, model.process(h)) for h in wl)
        out["model_hit_rate"] = round(hits / sum(len(h) for h in wl), 4)
        out["event_log_equal"] = model.events == [(k, h) for k, h in nat["events"]]
    bat = run_batch(wl, a.blocks, a.backend)
    out["native_batch"] = {"requests_per_s": round(a.requests / bat["seconds"], 1),
                           "blocks_per_s": round(bat["blocks"] / bat["seconds"], 1),
                           "hit_rate": round(bat["hit_rate"], 4),
                           "event_log_equal_to_handles": bat["events"] == nat["events"]}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()
