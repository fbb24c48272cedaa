"""Engine-level transfer benchmarks on one GPU (Llama-3-8B KV geometry).

Sections:

* ``offload`` - blocks pushed through the production offload path: the
  ``InstanceLeader`` enqueues G1 blocks, the G1->G2 pipeline (presence
  policy, batching) allocates, copies with the worker's transfer manager and
  registers them, and auto-chains G2->G3 onto the disk tier. Reports
  blocks/s and GB/s of each hop from wall time (the pipelines are
  host-driven), plus pipeline counters.
* ``bidir`` - G1->G2 and G2->G1 at the same time on two streams (each with
  half of the SMs), device time with CUDA events: PCIe in both directions.
* ``onboard`` - ``InstanceLeader.find_matches`` + ``onboard`` of a cached
  prefix (G2 hits copied to G1), launch-to-completion time of the onboard.

    python -m kvbm_b200.bench.engine_bench --blocks 512 --sections offload,bidir,onboard

Parity: crates/kvbm-engine/src/bin/bench_engine.rs (isolated / bidir /
offload-pipeline benches over the production leader and worker).
"""

from __future__ import annotations

import argparse
import json
import random
import tempfile
import time

import torch

from ..engine.leader import InstanceLeader, ParallelWorkers
from ..engine.offload import OffloadEngine, OffloadItem, OffloadPipeline, PresenceFilter, make_tier_executor
from ..engine.worker import Worker
from ..logical.manager import BlockManager, Tier
from ..logical.sequence import sequence_hashes
from ..ops import kv_ops
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig


def _g1(args, nb):
    cfg = LayoutConfig.for_model(nb, args.layers, args.heads, 128, 16)
    g1 = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD)
    g1._flat().random_(0, 256)
    return g1


def offload_section(args, out):
    n = args.blocks
    g1 = _g1(args, n + 8)
    with tempfile.TemporaryDirectory() as d:
        w = Worker(0, g1, g2_blocks=n + 8, g3_blocks=n + 8 if args.g3 else 0, g3_path=f"{d}/g3.bin")
        g2 = BlockManager(n + 8, 16, "lineage", Tier.G2)
        g3 = BlockManager(n + 8, 16, "lineage", Tier.G3, registry=g2.registry) if args.g3 else None
        eng = OffloadEngine()
        done23 = {"n": 0, "t": None}
        if g3 is not None:
            p23 = OffloadPipeline("g2_to_g3", g3, make_tier_executor(w.handles.g2, g3, w.handles.g3, w.tm),
                                  PresenceFilter(g3))
            eng.add(p23)

            def chain(blocks):
                h = p23.enqueue([OffloadItem(b.sequence_hash, b.block_id, b.clone()) for b in blocks])
                done23.setdefault("handles", []).append(h)
        else:
            chain = None
        p12 = OffloadPipeline("g1_to_g2", g2, make_tier_executor(w.handles.g1, g2, w.handles.g2, w.tm),
                              PresenceFilter(g2), on_registered=chain)
        p12.cfg.max_batch = args.batch
        eng.add(p12)
        leader = InstanceLeader(g2, ParallelWorkers([w]), g3=g3, offload=eng)
        # warm-up: a few blocks through both hops (first launches, streams, module loads)
        warm = sequence_hashes(list(range(10**6, 10**6 + 4 * 16)), 16)
        leader.offload_g1(warm, [0, 1, 2, 3]).wait(300)
        for hh in done23.pop("handles", []):
            hh.wait(300)
        for k in list(eng.pipelines.values()):
            k.stats.update({"submit_s": 0.0, "complete_s": 0.0})
        hashes = sequence_hashes(list(range(n * 16)), 16)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        h = leader.offload_g1(hashes, list(range(n)))
        state = h.wait(300)
        t1 = time.perf_counter()
        for hh in done23.get("handles", []):
            hh.wait(300)
        t2 = time.perf_counter()
        bpb = g1.config.bytes_per_block
        r = {"section": "offload", "blocks": n, "batch": args.batch, "state": state.value,
             "g1_to_g2_ms": round((t1 - t0) * 1e3, 2), "g1_to_g2_blocks_per_s": round(n / (t1 - t0)),
             "g1_to_g2_gbps": round(n * bpb / (t1 - t0) / 1e9, 2), "stats": eng.stats()}
        if g3 is not None:
            r.update({"g2_to_g3_done_ms": round((t2 - t0) * 1e3, 2),
                      "g1_to_g3_chain_gbps": round(n * bpb / (t2 - t0) / 1e9, 2)})
        out.append(r)
        print(json.dumps(r, default=str), flush=True)
        eng.close()


def bidir_section(args, out):
    n = args.blocks
    g1 = _g1(args, 2 * n + 8)
    cfg = g1.config
    g2 = KvLayout.allocate(LayoutConfig(**{**cfg.__dict__, "num_blocks": 2 * n + 8}), "fully_contiguous",
                           KvBlockLayout.OPERATIONAL_NHD, location="pinned")
    rng = random.Random(3)
    ids = rng.sample(range(2 * n + 8), 2 * n)
    a = torch.tensor(ids[:n], dtype=torch.int32, device="cuda")
    b = torch.tensor(ids[n:], dtype=torch.int32, device="cuda")
    half = max(1, kv_ops.sm_count() // 2)
    s_up, s_down = torch.cuda.Stream(), torch.cuda.Stream()
    main = torch.cuda.current_stream()

    def both():
        start = torch.cuda.Event()
        start.record(main)
        for s in (s_up, s_down):
            s.wait_event(start)
        kv_ops.kv_transfer(g1, a, g2, a, engine=args.engine, max_ctas=half, stream=s_down)  # offload
        kv_ops.kv_transfer(g2, b, g1, b, engine=args.engine, max_ctas=half, stream=s_up)    # onboard
        for s in (s_up, s_down):
            ev = torch.cuda.Event()
            ev.record(s)
            main.wait_event(ev)

    def one(src, dst, ids):
        kv_ops.kv_transfer(src, ids, dst, ids, engine=args.engine)

    bpb = cfg.bytes_per_block
    cases = (("d2h_only", lambda: one(g1, g2, a), n * bpb), ("h2d_only", lambda: one(g2, g1, b), n * bpb),
             ("bidir", both, 2 * n * bpb))
    for name, fn, nbytes in cases:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / args.iters
        r = {"section": "bidir", "case": name, "blocks": n, "engine": args.engine, "ms": round(ms, 3),
             "gbps": round(nbytes / ms / 1e6, 2)}
        out.append(r)
        print(json.dumps(r), flush=True)


def onboard_section(args, out):
    n = args.blocks
    g1 = _g1(args, 2 * n + 8)
    w = Worker(0, g1, g2_blocks=n + 8)
    g2 = BlockManager(n + 8, 16, "lineage", Tier.G2)
    leader = InstanceLeader(g2, ParallelWorkers([w]))
    hashes = sequence_hashes(list(range(n * 16)), 16)
    blocks = g2.allocate_blocks(n)
    kv_ops.kv_transfer(g1, list(range(n)), w.g2_layout, [x.block_id for x in blocks])
    for x in g2.register_mutable(blocks, hashes):
        x.release()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.warmup + args.iters):
        res = leader.find_matches(hashes)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()  # the onboard runs on the transfer manager's stream; e is recorded after it completed
        note = leader.onboard(res.g2_blocks, list(range(n, 2 * n)))
        note.wait()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
        res.release()
    ms = sorted(times[args.warmup:])[len(times[args.warmup:]) // 2]
    r = {"section": "onboard", "blocks": n, "matched": n, "ms": round(ms, 3),
         "gbps": round(n * g1.config.bytes_per_block / ms / 1e6, 2)}
    out.append(r)
    print(json.dumps(r), flush=True)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--blocks", type=int, default=512)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--engine", default="tile")
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--no-g3", dest="g3", action="store_false")
    p.add_argument("--sections", default="offload,bidir,onboard")
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    torch.cuda.set_device(0)
    out: list[dict] = []
    secs = a.sections.split(",")
    if "offload" in secs:
        offload_section(a, out)
    if "bidir" in secs:
        bidir_section(a, out)
    if "onboard" in secs:
        onboard_section(a, out)
    if a.out:
        with open(a.out, "w") as f:
            for r in out:
                f.write(json.dumps(r, default=str) + "\n")


if __name__ == "__main__":
    main()
