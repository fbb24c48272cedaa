"""KV transfer bandwidth microbenchmark (the counterpart of the reference's
``kvbench`` example, crates/kvbm-kernels/examples/kvbench.rs).

Measures G1->G2 (offload), G2->G1 (onboard) and G1->G1 (transform) block
copies on the Llama KV geometry with seed-random non-contiguous block ids,
for the SM kernels (``tile``: warp-per-tile direct loads; ``tma``: bulk
async copies staged through shared memory) and for the copy-engine baseline
(one cudaMemcpyAsync per contiguous region). Device time from CUDA events
on the launching stream, after warm-up, with an L2 flush (a 256 MiB write)
before each timed iteration.

    python -m kvbm_b200.bench.kvbench --layers 32 --heads 8 --batches 1,8,64,512
"""

from __future__ import annotations

import argparse
import json
import random

import torch

from ..ops import kv_ops
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig

L2_FLUSH_BYTES = 256 << 20


def _time(fn, iters: int, warmup: int, flush: torch.Tensor) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.fill_(1)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def _ce_regions(src: KvLayout, s_ids, dst: KvLayout, d_ids):
    """Contiguous regions for the copy-engine baseline."""
    if src.kind == dst.kind == "fully_contiguous" and src.block_layout == dst.block_layout:
        bpb = src.config.bytes_per_block
        return ([src.layer_base(0) + b * src.block_stride for b in s_ids],
                [dst.layer_base(0) + b * dst.block_stride for b in d_ids], bpb)
    sp, dp = [], []
    c = src.config
    for sb, db in zip(s_ids, d_ids):
        for l in range(c.num_layers):
            for o in range(c.outer_dim):
                sp.append(src.memory_region(sb, l, o)[0])
                dp.append(dst.memory_region(db, l, o)[0])
    return sp, dp, c.bytes_per_chunk


# on-device engines: tile (pipelined cast kernel, every conversion in hardware), tile_sw1 / tile_sw2 /
# tile_sw (a quarter, half or all of its bf16 <-> fp8 conversions on the integer / FMA pipes; the
# library default is none for quantise, a quarter for dequantise), tile1 (one tile at a time), tma
CAST_ENGINES = ("tile", "tile_sw1", "tile_sw2", "tile_sw", "tile1", "tma")


def run(args) -> list[dict]:
    torch.cuda.set_device(0)
    rng = random.Random(args.seed)
    batches = [int(x) for x in args.batches.split(",")]
    nmax = max(batches)
    pool_blocks = max(2 * nmax, 64)
    cfg = LayoutConfig.for_model(pool_blocks, args.layers, args.heads, args.head_dim, args.page)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    nhd = KvBlockLayout.OPERATIONAL_NHD
    layouts = {
        "fc": lambda loc: KvLayout.allocate(cfg, "fully_contiguous", nhd, location=loc),
        "lw": lambda loc: KvLayout.allocate(cfg, "layer_separate", nhd, location=loc),
    }
    results = []
    sections = set(args.sections.split(","))
    for g1_kind in (args.layouts.split(",") if "g12" in sections else []):
        g1 = layouts[g1_kind]("device")
        g2 = KvLayout.allocate(cfg, "fully_contiguous", nhd, location="pinned")
        g1._flat().random_(0, 256)
        for n in batches:
            s_ids = rng.sample(range(pool_blocks), n)
            d_ids = rng.sample(range(pool_blocks), n)
            sid = torch.tensor(s_ids, dtype=torch.int32, device="cuda")
            did = torch.tensor(d_ids, dtype=torch.int32, device="cuda")
            nbytes = n * cfg.bytes_per_block
            for direction, (a, ai, b, bi) in {"g1_to_g2": (g1, sid, g2, did), "g2_to_g1": (g2, did, g1, sid)}.items():
                for engine in args.engines.split(","):
                    if engine == "ce":
                        sp, dp, sz = _ce_regions(a, ai.tolist(), b, bi.tolist())
                        fn = lambda sp=sp, dp=dp, sz=sz: kv_ops.memcpy_pairs_ce(sp, dp, sz)
                    elif engine == "ce_graph":
                        # the same copy-engine regions captured once as a graph of memcpy nodes, replayed
                        sp, dp, sz = _ce_regions(a, ai.tolist(), b, bi.tolist())
                        g = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(g, capture_error_mode="thread_local"):
                            kv_ops.memcpy_pairs_ce(sp, dp, sz, stream=torch.cuda.current_stream())
                        fn = g.replay
                    else:
                        fn = lambda a=a, ai=ai, b=b, bi=bi, engine=engine: kv_ops.kv_transfer(
                            a, ai, b, bi, engine=engine, max_ctas=args.max_ctas)
                    ms = _time(fn, args.iters, args.warmup, flush)
                    r = {"direction": direction, "g1_layout": g1_kind, "blocks": n, "bytes": nbytes,
                         "engine": engine, "ms": round(ms, 4), "gbps": round(nbytes / ms / 1e6, 2)}
                    results.append(r)
                    print(json.dumps(r), flush=True)
        del g1, g2
    if "d2d" not in sections:
        return results
    # device-local transform (HND <- NHD) and copy, HBM bound
    a = KvLayout.allocate(cfg, "fully_contiguous", nhd)
    a._flat().random_(0, 256)
    n = nmax
    s_ids = torch.tensor(rng.sample(range(pool_blocks), n), dtype=torch.int32, device="cuda")
    d_ids = torch.tensor(rng.sample(range(pool_blocks), n), dtype=torch.int32, device="cuda")
    cfg8 = LayoutConfig.for_model(pool_blocks, args.layers, args.heads, args.head_dim, args.page, torch.float8_e4m3fn)
    dsts = {
        "g1_to_g1_nhd_to_hnd": KvLayout.allocate(cfg, "layer_separate", KvBlockLayout.OPERATIONAL_HND),
        "g1_to_g1_copy": KvLayout.allocate(cfg, "fully_contiguous", nhd),
        "g1_to_g1_universal": KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.UNIVERSAL),
        # bf16 -> fp8 e4m3 with one fp32 scale per (block, layer, K/V, head), NHD -> HND
        "g1_to_g1_fp8_quant": KvLayout.allocate(cfg8, "fully_contiguous", KvBlockLayout.OPERATIONAL_HND,
                                                fp8_scales=True),
    }
    for name, b in dsts.items():
        if args.d2d and name not in args.d2d.split(","):
            continue
        for engine in [e for e in CAST_ENGINES if e in args.engines.split(",")]:
            # tile1: the fp8 casts on the one-tile-at-a-time kernel (tile: the pipelined one; tile_sw:
            # the pipelined one converting on the integer / FMA pipes)
            kv_ops.set_cast_pipeline(engine != "tile1")
            sq = {"tile_sw1": 1, "tile_sw2": 2, "tile_sw": 4}.get(engine, 0)
            kv_ops.set_cast_softconv(sq, sq)
            eng = "tile" if engine.startswith("tile") else engine
            ms = _time(lambda: kv_ops.kv_transfer(a, s_ids, b, d_ids, engine=eng), args.iters, args.warmup,
                       flush)
            nbytes = n * cfg.bytes_per_block
            moved = nbytes + n * b.config.bytes_per_block  # read + write (fp8 writes half)
            r = {"direction": name, "blocks": n, "bytes": nbytes, "engine": engine,
                 "ms": round(ms, 4), "gbps_rw": round(moved / ms / 1e6, 2)}
            results.append(r)
            print(json.dumps(r), flush=True)
        if name == "g1_to_g1_fp8_quant":
            back = KvLayout.allocate(cfg, "fully_contiguous", nhd)
            for engine in [e for e in CAST_ENGINES if e in args.engines.split(",")]:
                kv_ops.set_cast_pipeline(engine != "tile1")
                # tile / tile1: the dequantiser's default share; tile_sw*: that share of the conversions
                kv_ops.set_cast_softconv(None, {"tile_sw1": 1, "tile_sw2": 2, "tile_sw": 4}.get(engine))
                eng = "tile" if engine.startswith("tile") else engine
                ms = _time(lambda: kv_ops.kv_transfer(b, d_ids, back, s_ids, engine=eng), args.iters,
                           args.warmup, flush)
                nbytes = n * cfg.bytes_per_block
                moved = nbytes + n * b.config.bytes_per_block
                r = {"direction": "g1_to_g1_fp8_dequant", "blocks": n, "bytes": nbytes, "engine": engine,
                     "ms": round(ms, 4), "gbps_rw": round(moved / ms / 1e6, 2)}
                results.append(r)
                print(json.dumps(r), flush=True)
        kv_ops.set_cast_pipeline(True)
        kv_ops.set_cast_softconv()
        if name == "g1_to_g1_copy" and "ce" in args.engines.split(","):
            src_p = [a.layer_base(0) + int(x) * a.block_stride for x in s_ids.tolist()]
            dst_p = [b.layer_base(0) + int(x) * b.block_stride for x in d_ids.tolist()]
            sp = torch.tensor(src_p, dtype=torch.int64, device="cuda")
            dp = torch.tensor(dst_p, dtype=torch.int64, device="cuda")
            for engine, fn in {
                "copy_pairs": lambda: kv_ops.copy_pairs(sp, dp, cfg.bytes_per_block, align=16),
                "ce": lambda: kv_ops.memcpy_pairs_ce(src_p, dst_p, cfg.bytes_per_block),
            }.items():
                ms = _time(fn, args.iters, args.warmup, flush)
                nbytes = n * cfg.bytes_per_block
                r = {"direction": name, "blocks": n, "bytes": nbytes, "engine": engine,
                     "ms": round(ms, 4), "gbps_rw": round(2 * nbytes / ms / 1e6, 2)}
                results.append(r)
                print(json.dumps(r), flush=True)
    return results


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--page", type=int, default=16)
    p.add_argument("--batches", default="1,8,64,512")
    p.add_argument("--layouts", default="fc,lw")
    p.add_argument("--engines", default="tile,tma,ce", help="tile, tile1, tma, ce, ce_graph")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--max-ctas", type=int, default=0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--sections", default="g12,d2d", help="g12 (G1<->G2), d2d (on-device transforms)")
    p.add_argument("--d2d", default="", help="subset of d2d cases (comma list); empty = all")
    p.add_argument("--out", default=None)
    args = p.parse_args(argv)
    res = run(args)
    if args.out:
        with open(args.out, "w") as f:
            for r in res:
                f.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()
