"""Decode-projection GEMM microbenchmark: the tcgen05 skinny GEMM against
cuBLAS (``torch.matmul``) on Llama-3-8B's weight shapes for a few batch rows.

For each shape, R copies of the weight (together >= 512 MiB, so no copy is
still in the 126 MB L2 when its turn comes again) are multiplied in turn,
``launches`` GEMMs captured in one CUDA graph; the graph is replayed and
timed with CUDA events, and the time per launch is the replay time over the
launch count. This removes host launch overhead and the event timer's ~2 us
granularity from single-launch timings, and mirrors the decode step, where
projections run back to back from a graph. The figure of merit is the weight
bytes per second against the measured copy bandwidth.

    python -m kvbm_b200.bench.gemm_bench --batch 1,8,32,64,128 [--modes auto,streamk,cluster]
"""

from __future__ import annotations

import argparse
import json

import torch

from ..ops import llama_ops

# (name, N, K): one tile (fixed per-launch cost), an 8 MiB weight, then Llama-3-8B's fused q/k/v,
# o, fused gate/up, down and lm_head
SHAPES = [("tiny", 128, 64), ("small", 1024, 4096), ("qkv", 6144, 4096), ("o", 4096, 4096),
          ("gate_up", 28672, 4096), ("down", 4096, 14336), ("lm_head", 128256, 4096)]


def _graph_time(step, launches: int, replays: int) -> float:
    """Milliseconds per launch of a captured sequence of ``launches`` GEMMs."""
    step()  # warm: workspace, kernel attributes, cuBLAS heuristics
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(replays):
        g.replay()
    e.record()
    e.synchronize()
    del g
    return s.elapsed_time(e) / (replays * launches)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--batch", default="1,8,32,64,128")
    p.add_argument("--shapes", default=",".join(n for n, _, _ in SHAPES[2:]))
    p.add_argument("--launches", type=int, default=24, help="GEMM launches per captured graph")
    p.add_argument("--replays", type=int, default=5)
    p.add_argument("--ctas", default="0", help="comma list of persistent CTA counts to try (0 = one per SM)")
    p.add_argument("--modes", default="auto", help="comma list of skinny-GEMM modes: auto, streamk, cluster")
    p.add_argument("--timeline", action="store_true",
                   help="also print per-phase %%globaltimer stamps of one stream-K launch (after one on another copy)")
    args = p.parse_args(argv)
    torch.cuda.set_device(0)
    want = set(args.shapes.split(","))
    for name, N, K in SHAPES:
        if name not in want:
            continue
        wbytes = N * K * 2
        R = max(2, -(-(512 << 20) // wbytes))
        ws = [(torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5).to(torch.bfloat16)
              for _ in range(R)]
        n = max(args.launches, R)
        for M in (int(b) for b in args.batch.split(",")):
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            ref = x.float() @ ws[-1].float().t()

            def cublas():
                for i in range(n):
                    torch.matmul(x, ws[i % R].t(), out=out)

            t_cublas = _graph_time(cublas, n, args.replays)
            row = {"shape": name, "M": M, "N": N, "K": K, "copies": R, "cublas_us": round(t_cublas * 1e3, 2),
                   "cublas_gbs": round(wbytes / t_cublas / 1e6, 1)}
            runs = [(m, nc) for m in args.modes.split(",") for nc in (int(v) for v in args.ctas.split(","))
                    if nc == 0 or m == "streamk"]
            for mode, nc in runs:
                llama_ops.set_skinny_gemm_mode(mode)

                def tc():
                    for i in range(n):
                        llama_ops.skinny_gemm(x, ws[i % R], out=out, ctas=nc)

                t = _graph_time(tc, n, args.replays)
                llama_ops.skinny_gemm(x, ws[-1], out=out, ctas=nc)
                torch.cuda.synchronize()
                err = (out.float() - ref).abs().max().item()
                key = f"{mode}{nc or ''}"
                row[key + "_us"] = round(t * 1e3, 2)
                row[key + "_gbs"] = round(wbytes / t / 1e6, 1)
                row[key + "_maxerr"] = round(err, 4)
            llama_ops.set_skinny_gemm_mode("auto")
            if args.timeline:
                llama_ops.set_skinny_gemm_mode("streamk")

                def two():
                    llama_ops.skinny_gemm(x, ws[0], out=out)
                    llama_ops.skinny_gemm(x, ws[1], out=out)

                two()
                torch.cuda.synchronize()
                llama_ops.skinny_gemm(x, ws[0], out=out)  # the stamped launch follows this one
                row["timeline_us"] = llama_ops.skinny_gemm_timeline(lambda: llama_ops.skinny_gemm(x, ws[1], out=out))
                llama_ops.set_skinny_gemm_mode("auto")
            row["status"] = llama_ops.skinny_gemm_status()
            print(json.dumps(row), flush=True)
        del ws


if __name__ == "__main__":
    main()
