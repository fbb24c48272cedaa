"""One-to-many G1 fan-out across the GPUs of one node: NVSwitch multicast
(``multimem.st``, one store per 16 bytes reaches every rank) against the
per-peer NVLink push (rank 0 stores into each peer in turn) and the NCCL
broadcast baseline (gather, ``broadcast``, scatter).

Geometry: Llama-3-8B KV (32 layers, 8 KV heads, head_dim 128, page 16,
bf16: 2 MiB per block). Rank 0 fans ``--blocks`` blocks out to every rank.
Each iteration is timed with CUDA events on every rank's stream (rank 0's
launch to each rank's completion wait) after a barrier; the reported time is
the median over iterations of the max over ranks. ``delivered_gbps`` counts
the bytes that land in the other ranks (blocks x block bytes x (N - 1)) per
second; ``per_peer_gbps`` the bytes one peer receives per second.

    torchrun --nproc-per-node N -m kvbm_b200.bench.fanout_bench
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
from datetime import timedelta

import torch
import torch.distributed as dist

from ..parallel.collectives import NcclCollectives, NvlsFanoutCollectives, NvlsUnavailable, P2PFanoutCollectives
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig


def _time(coll, src, dst, iters: int, warmup: int) -> float:
    times = []
    for it in range(warmup + iters):
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        coll.broadcast(src, dst)
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b)], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        if it >= warmup:
            times.append(float(ms.item()))
    if hasattr(coll, "check"):
        coll.check()
    return statistics.median(times)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--pool-blocks", type=int, default=320)
    p.add_argument("--blocks", type=int, default=256)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--paths", default="nvls,p2p,nccl")
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    cfg = LayoutConfig.for_model(a.pool_blocks, 32, 8, 128, 16)
    src = list(range(a.blocks))
    dst = list(range(a.pool_blocks - a.blocks, a.pool_blocks))
    nbytes = a.blocks * cfg.bytes_per_block
    line = {"bench": "fanout", "n_gpus": world, "blocks": a.blocks, "bytes": nbytes, "geometry": "llama3_8b",
            "timing": "median over iterations of max over ranks, CUDA events"}
    for path in a.paths.split(","):
        if path == "nvls":
            g1, handle, off = NvlsFanoutCollectives.allocate_pool(cfg)
            try:
                coll = NvlsFanoutCollectives(g1, handle, off, wait_ns=20_000_000_000)
            except NvlsUnavailable as e:
                line["nvls"] = {"unavailable": str(e)}
                continue
        else:
            g1 = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, zero=True)
            coll = P2PFanoutCollectives(g1) if path == "p2p" else NcclCollectives(g1, max_blocks=64)
        ms = _time(coll, src, dst, a.iters, a.warmup)
        line[path] = {"ms": round(ms, 3), "delivered_gbps": round(nbytes * (world - 1) / ms / 1e6, 1),
                      "per_peer_gbps": round(nbytes / ms / 1e6, 1)}
        del coll, g1
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
        if a.out:
            with open(a.out, "a") as f:
                f.write(json.dumps(line) + "\n")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
