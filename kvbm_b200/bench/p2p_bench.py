"""Isolated prefill -> decode KV transfer over NVLink (2 ranks, one box).

Rank 0 (prefill) maps rank 1's (decode) paged G1 pool through CUDA IPC and
moves whole requests' KV (all layers, non-contiguous block ids on both
sides) with the fused transfer kernel, nothing else running. Baselines on
the same bytes:

* ``nccl_contig``: one NCCL send/recv of a contiguous buffer (the bus
  ceiling NCCL reaches, without any paging);
* ``nccl_paged``: what a NCCL-based P->D path has to do with paged KV -
  gather the blocks into a staging buffer, send/recv, scatter on the decode
  side (gather/scatter done with the same SM kernel).

Device time with CUDA events (max over the two ranks), L2 flushed before
every timed iteration. Roofline: the peer copy bandwidth measured first in
the same run (``peer_copy`` rows: a 1 GiB ``cudaMemcpyAsync`` from this
GPU's memory into the peer's, the copy engines' path, and the same bytes by
the SM copy kernel; median of ``--peer-iters``); fractions are reported
against the best of those and against the 900 GB/s nominal NVLink 5 rate.

    torchrun --nproc-per-node 2 -m kvbm_b200.bench.p2p_bench
"""

from __future__ import annotations

import argparse
import json
import os
import random
from datetime import timedelta

import torch
import torch.distributed as dist

from ..ops import kv_ops
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig, LayoutDescriptor

NVLINK_NOMINAL_GBPS = 900.0
PEER_COPY_GBPS = 770.0  # replaced by the run's own measurement in main()


def measure_peer_copy(rank, remote_ptr, nbytes, iters, gloo) -> list[dict]:
    """1 GiB from this GPU into the peer's memory: copy engine (cudaMemcpyAsync over UVA) and the SM copy
    kernel; device time with CUDA events, median of ``iters`` after warm-up."""
    dev = torch.device("cuda", rank)
    src = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    src.random_(0, 256)
    out = []
    for path in ("cudaMemcpyAsync_peer", "sm_copy_kernel_peer"):
        def fn(path=path):
            if rank != 0:
                return
            if path.startswith("cudaMemcpy"):
                from ..ops import _lib
                _lib.check(_lib.load().kvbm_memcpy_async(remote_ptr, src.data_ptr(), nbytes, None), "memcpy")
            else:
                kv_ops.copy_pairs([src.data_ptr()], [remote_ptr], nbytes)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            dist.barrier(group=gloo)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        ms = sorted(ts)[len(ts) // 2]
        both = [None, None]
        dist.all_gather_object(both, ms, group=gloo)
        r = {"path": "peer_copy", "how": path, "bytes": nbytes, "ms": round(both[0], 4),
             "gbps": round(nbytes / both[0] / 1e6, 1), "iters": iters,
             "frac_of_nominal": round(nbytes / both[0] / 1e6 / NVLINK_NOMINAL_GBPS, 3)}
        out.append(r)
        if rank == 0:
            print(json.dumps(r), flush=True)
    return out


def gloo_of(args):
    return args._gloo


def rope_push_section(args, rank, local, remote, cfg, pool_blocks, timed, rng) -> list[dict]:
    """One prefill's worth of layers (``--blocks`` x 16 tokens, 32 query / ``--heads`` KV heads):
    the RoPE/KV kernel stores every layer's K/V into the peer's pool."""
    from ..ops import llama_ops

    T = args.blocks * 16
    hq = 4 * args.heads
    out = []
    dev = torch.device("cuda", rank)
    qkv = torch.randn(T, hq + 2 * args.heads, 128, device=dev, dtype=torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float64) / 128))
    f = torch.outer(torch.arange(T, dtype=torch.float64), inv)
    cs = torch.cat([f.cos(), f.sin()], dim=-1).float().to(dev)
    d_blocks = torch.tensor(rng.sample(range(pool_blocks), args.blocks), dtype=torch.long, device=dev)
    rslots = d_blocks[pos.long() // 16] * 16 + pos.long() % 16
    hog_a = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    hog_b = torch.empty_like(hog_a)
    nbytes = T * 2 * args.heads * 128 * 2 * args.layers
    cases = [("kv", False, 4), ("kv", True, 4), ("all", False, 4)] + [
        (h, False, u) for u in args.rope_unrolls for h in ("kv", "all") if u != 4]
    for heads, busy, unroll in cases:
        llama_ops.set_rope_unroll(unroll)

        def fn():
            if rank == 0:
                for l in range(args.layers):
                    rk = remote.layer_base(l)
                    llama_ops.rope_kv_push(qkv, pos, cs, hq, args.heads, None,
                                           (rk, rk + remote.outer_stride, remote.block_stride, remote.token_stride,
                                            remote.head_stride, 16, rslots), heads=heads)
            elif busy:
                for _ in range(24):  # ~8 ms of 1 GiB copies: the decode GPU's HBM stays loaded meanwhile
                    hog_b.copy_(hog_a)
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.iters):
            dist.barrier(group=gloo_of(args))
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        both = [None, None]
        dist.all_gather_object(both, sorted(ts)[len(ts) // 2], group=gloo_of(args))
        ms = both[0]  # the pushing rank's device time
        r = {"path": "rope_push", "heads": heads, "unroll": unroll, "decode_gpu": "streaming_hbm" if busy else "idle",
             "tokens": T,
             "layers": args.layers, "bytes": nbytes, "ms": round(ms, 4), "gbps": round(nbytes / ms / 1e6, 1),
             "frac_of_peer_copy": round(nbytes / ms / 1e6 / PEER_COPY_GBPS, 3)}
        out.append(r)
        if rank == 0:
            print(json.dumps(r), flush=True)
    llama_ops.set_rope_unroll(4)
    # copy-engine baseline: the RoPE kernel writes K/V into a local per-layer staging area, then one
    # cudaMemcpy2DAsync per layer moves the request's rows (K+V of one layer of a block are adjacent
    # in the fully contiguous layout) into consecutive destination blocks of the peer pool
    bpl = 2 * 16 * args.heads * 128 * 2  # K+V bytes of one layer of one block
    staging = torch.empty(args.layers * args.blocks * bpl, dtype=torch.uint8, device=dev)
    first = pool_blocks - args.blocks

    def ce():
        if rank == 0:
            for l in range(args.layers):
                kv_ops.memcpy_2d_ce(remote.layer_base(l) + first * remote.block_stride, remote.block_stride,
                                    staging.data_ptr() + l * args.blocks * bpl, bpl, bpl, args.blocks)

    for _ in range(args.warmup):
        ce()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.iters):
        dist.barrier(group=gloo_of(args))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        ce()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    both = [None, None]
    dist.all_gather_object(both, sorted(ts)[len(ts) // 2], group=gloo_of(args))
    ms = both[0]
    r = {"path": "ce_2d_per_layer", "tokens": T, "layers": args.layers, "bytes": nbytes, "ms": round(ms, 4),
         "gbps": round(nbytes / ms / 1e6, 1), "frac_of_peer_copy": round(nbytes / ms / 1e6 / PEER_COPY_GBPS, 3),
         "note": "copy engines only; needs the K/V staged locally first and consecutive destination blocks"}
    out.append(r)
    if rank == 0:
        print(json.dumps(r), flush=True)
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--blocks", type=int, default=512, help="blocks per request (512 = 8192 tokens)")
    p.add_argument("--requests", default="1,4")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--engines", default="tile,tma")
    p.add_argument("--ctas", default="0,32,64")
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--dst-layout", default="nhd", choices=["nhd", "hnd"])
    p.add_argument("--rope-push", action="store_true",
                   help="also time the fused RoPE + KV push kernel (the bench's prefill path), with the decode "
                        "GPU idle and with it streaming HBM (a stand-in for decode)")
    p.add_argument("--rope-unrolls", default="2,8", help="extra RoPE/KV kernel unroll depths to time")
    p.add_argument("--peer-iters", type=int, default=10)
    p.add_argument("--bulk-peer", action="store_true",
                   help="also time the TMA bulk copy storing into the peer's pool (TMA stores to NVLink memory)")
    p.add_argument("--src-heads", type=int, default=0,
                   help="heterogeneous-TP shape: the pushing pool holds this many KV heads and stores them at "
                        "--head-offset of the decode pool's --heads heads (0: same heads on both sides)")
    p.add_argument("--head-offset", type=int, default=0)
    p.add_argument("--out", default=None)
    args = p.parse_args(argv)
    args.rope_unrolls = [int(x) for x in args.rope_unrolls.split(",") if x]
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    assert world == 2
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", rank))
    gloo = dist.new_group(backend="gloo")
    args._gloo = gloo
    reqs = [int(x) for x in args.requests.split(",")]
    nmax = max(reqs) * args.blocks
    pool_blocks = 2 * nmax + 8
    sh = args.src_heads or args.heads
    cfg = LayoutConfig.for_model(pool_blocks, args.layers, sh if rank == 0 else args.heads, 128, 16)
    nhd = KvBlockLayout.OPERATIONAL_NHD
    dst_bl = nhd if args.dst_layout == "nhd" else KvBlockLayout.OPERATIONAL_HND
    local = KvLayout.allocate(cfg, "fully_contiguous", nhd if rank == 0 else dst_bl)
    hkw = {"dst_head_offset": args.head_offset, "num_heads": sh} if args.src_heads else {}
    local._flat().random_(0, 256)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    # exchange pools
    descs = [None, None]
    dist.all_gather_object(descs, local.descriptor().to_dict(), group=gloo)
    remote = KvLayout.from_descriptor(LayoutDescriptor.from_dict(descs[1])) if rank == 0 else None
    rng = random.Random(7)
    results = []
    global PEER_COPY_GBPS
    pc = measure_peer_copy(rank, remote.base_ptr if rank == 0 else 0, 1 << 30, args.peer_iters, gloo)
    results += pc
    PEER_COPY_GBPS = max(r["gbps"] for r in pc)

    def timed(fn) -> float:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        ts = []
        for _ in range(args.iters):
            flush.fill_(1)
            dist.barrier(group=gloo)
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        ts.sort()
        mine = ts[len(ts) // 2]
        both = [None, None]
        dist.all_gather_object(both, mine, group=gloo)
        return max(both)

    for nreq in reqs:
        n = nreq * args.blocks
        s_ids = torch.tensor(rng.sample(range(pool_blocks), n), dtype=torch.int32, device="cuda")
        d_ids = torch.tensor(rng.sample(range(pool_blocks), n), dtype=torch.int32, device="cuda")
        nbytes = n * cfg.bytes_per_block
        engines = args.engines.split(",") + (["tma_bulk_peer"] if args.bulk_peer else [])
        for engine in engines:
            for ctas in [int(c) for c in args.ctas.split(",")]:
                ran = [None]

                def fn(engine=engine, ctas=ctas):
                    if rank == 0:
                        if engine == "tma_bulk_peer":
                            ran[0] = kv_ops.kv_transfer(local, s_ids, remote, d_ids, engine="tma", max_ctas=ctas,
                                                        bulk=True, **hkw)
                        else:
                            ran[0] = kv_ops.kv_transfer(local, s_ids, remote, d_ids, engine=engine, max_ctas=ctas,
                                                        **hkw)
                ms = timed(fn)
                r = {"path": f"fused_{engine}", "kernel": ran[0], "max_ctas": ctas, "requests": nreq,
                     "heads": f"{sh}->{args.heads}@{args.head_offset}" if args.src_heads else args.heads,
                     "bytes": nbytes, "ms": round(ms, 4), "gbps": round(nbytes / ms / 1e6, 1),
                     "frac_of_peer_copy": round(nbytes / ms / 1e6 / PEER_COPY_GBPS, 3),
                     "frac_of_nominal": round(nbytes / ms / 1e6 / NVLINK_NOMINAL_GBPS, 3)}
                results.append(r)
                if rank == 0:
                    print(json.dumps(r), flush=True)
        # correctness of the last fused transfer: compare a sample of blocks
        torch.cuda.synchronize()
        dist.barrier(group=gloo)
        sample = list(range(0, n, max(1, n // 16)))
        if rank == 0:
            data = local.gather_blocks(s_ids[sample].tolist()).cpu()
            dist.send(data.view(torch.uint8).reshape(-1), dst=1, group=gloo)
        else:
            got = local.gather_blocks(d_ids[sample].tolist()).cpu()
            if args.src_heads:  # [n, L, O, T, H, D]: the pushed heads only
                got = got[..., args.head_offset: args.head_offset + sh, :].contiguous()
            ref = torch.empty_like(got.view(torch.uint8).reshape(-1))
            dist.recv(ref, src=0, group=gloo)
            ok = torch.equal(got.view(torch.uint8).reshape(-1), ref)
            print(json.dumps({"check": "fused_transfer_exact", "requests": nreq, "ok": bool(ok)}), flush=True)
        if args.src_heads:
            continue  # the NCCL baselines move whole blocks of one geometry
        # NCCL baselines
        contig = torch.empty(nbytes, dtype=torch.uint8, device="cuda")

        def nccl_contig():
            if rank == 0:
                dist.send(contig, dst=1)
            else:
                dist.recv(contig, src=0)
        ms = timed(nccl_contig)
        r = {"path": "nccl_contig", "requests": nreq, "bytes": nbytes, "ms": round(ms, 4),
             "gbps": round(nbytes / ms / 1e6, 1), "frac_of_peer_copy": round(nbytes / ms / 1e6 / PEER_COPY_GBPS, 3)}
        results.append(r)
        if rank == 0:
            print(json.dumps(r), flush=True)
        staging = KvLayout.over_tensor(LayoutConfig.for_model(n, args.layers, args.heads, 128, 16), contig)
        seq_ids = torch.arange(n, dtype=torch.int32, device="cuda")

        def nccl_paged():
            if rank == 0:
                kv_ops.kv_transfer(local, s_ids, staging, seq_ids)
                dist.send(contig, dst=1)
            else:
                dist.recv(contig, src=0)
                kv_ops.kv_transfer(staging, seq_ids, local, d_ids)
        ms = timed(nccl_paged)
        r = {"path": "nccl_paged", "requests": nreq, "bytes": nbytes, "ms": round(ms, 4),
             "gbps": round(nbytes / ms / 1e6, 1), "frac_of_peer_copy": round(nbytes / ms / 1e6 / PEER_COPY_GBPS, 3)}
        results.append(r)
        if rank == 0:
            print(json.dumps(r), flush=True)
        del contig, staging
    if args.rope_push:
        results += rope_push_section(args, rank, local, remote, cfg, pool_blocks, timed, rng)
    if rank == 0 and args.out:
        with open(args.out, "w") as f:
            for r in results:
                f.write(json.dumps(r) + "\n")
    dist.barrier(group=gloo)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
