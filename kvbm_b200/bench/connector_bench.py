"""CPU cost of the connector's scheduler hooks per engine step (no GPU).

The scheduler-side connector runs inside the serving engine's scheduling
loop, so its per-step work adds to every step's latency. This bench drives a
``ConnectorLeader`` the way vLLM's scheduler does and times the hooks on the
host:

* **admission** - a wave of ``--requests`` new requests with
  ``--prompt``-token prompts: ``get_num_new_matched_tokens`` +
  ``update_state_after_alloc`` per request, then one ``build_connector_meta``
  for the prefill step (every full prompt block offloaded G1 -> G2) and the
  workers' report that registers the G2 blocks;
* **decode steps** - every request gains one token per step
  (``build_connector_meta`` + ``update_connector_output``); a block boundary
  every 16 steps offloads one block per request;
* **warm admission** - the same prompts again: prefix matches in G2 and
  onboard ops.

Reported: microseconds per step (median and p99) and per request. Timing is
``time.perf_counter_ns`` around the hook calls only.

    python -m kvbm_b200.bench.connector_bench [--requests 32,256] [--prompt 2048] [--steps 256]
"""

from __future__ import annotations

import argparse
import json
import time

import numpy as np

from ..connector.leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
from ..engine.leader import InstanceLeader
from ..logical.manager import BlockManager, Tier

BS = 16


def _pct(xs, q):
    return float(np.percentile(np.asarray(xs, dtype=np.float64), q))


def run(requests: int, prompt: int, steps: int, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    blocks_per_req = (prompt + steps) // BS + 2
    g2 = BlockManager(requests * blocks_per_req * 2 + 64, BS, "lineage", Tier.G2)
    L = ConnectorLeader(InstanceLeader.scheduler_side(g2), BS)
    prompts = [rng.integers(0, 128000, prompt).tolist() for _ in range(requests)]
    g1_next = [0]

    def alloc(n):
        ids = list(range(g1_next[0], g1_next[0] + n))
        g1_next[0] += n
        return ids

    def admit(tag):
        t0 = time.perf_counter_ns()
        sched = {}
        for i, p in enumerate(prompts):
            rid = f"{tag}{i}"
            L.create_slot(KvbmRequest(rid, p))
            n, _ = L.get_num_new_matched_tokens(rid, 0)
            ids = alloc(blocks_per_req)
            L.update_state_after_alloc(rid, ids, n or 0)
            sched[rid] = ([], [], prompt)
        meta = L.build_connector_meta(SchedulerOutputLite(1, sched))
        t1 = time.perf_counter_ns()
        L.update_connector_output(finished_sending=set(), finished_recving={f"{tag}{i}" for i in range(requests)},
                                  worker_meta={"offloaded": {1: 1}})
        t2 = time.perf_counter_ns()
        return (t1 - t0) / 1e3, (t2 - t1) / 1e3, len(meta)

    adm_us, rep_us, meta_bytes = admit("a")
    step_us = []
    tok = rng.integers(0, 128000, (steps, requests))
    for s in range(steps):
        sched = {f"a{i}": ([int(tok[s, i])], [], prompt + s + 1) for i in range(requests)}
        t0 = time.perf_counter_ns()
        L.build_connector_meta(SchedulerOutputLite(2 + s, sched))
        L.update_connector_output(finished_sending=set(), finished_recving=set(), worker_meta={"offloaded": {2 + s: 1}})
        step_us.append((time.perf_counter_ns() - t0) / 1e3)
    for i in range(requests):
        L.request_finished(f"a{i}")
    warm_us, _, warm_bytes = admit("b")
    return {"bench": "connector_cpu", "requests": requests, "prompt_tokens": prompt, "decode_steps": steps,
            "admission_us": round(adm_us, 1), "admission_us_per_request": round(adm_us / requests, 2),
            "register_report_us": round(rep_us, 1), "admission_meta_bytes": meta_bytes,
            "decode_step_us_p50": round(_pct(step_us, 50), 1), "decode_step_us_p99": round(_pct(step_us, 99), 1),
            "decode_step_us_per_request": round(_pct(step_us, 50) / requests, 3),
            "warm_admission_us": round(warm_us, 1), "warm_admission_us_per_request": round(warm_us / requests, 2),
            "warm_meta_bytes": warm_bytes, "g2_hits": L.leader.stats.get("g2_hits", 0)}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--requests", default="32,256")
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    for r in [int(x) for x in a.requests.split(",")]:
        line = run(r, a.prompt, a.steps)
        print(json.dumps(line), flush=True)
        if a.out:
            with open(a.out, "a") as f:
                f.write(json.dumps(line) + "\n")


if __name__ == "__main__":
    main()
