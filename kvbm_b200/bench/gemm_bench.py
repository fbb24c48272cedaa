"""Decode-projection GEMM microbenchmark: the tcgen05 skinny GEMM against
cuBLAS (``torch.matmul``) on Llama-3-8B's weight shapes for a few batch rows.

Each iteration first reads a 256 MiB buffer (L2 flush: the weights of one
projection fit in the 126 MB L2; a read leaves no dirty lines whose write-back
would compete with the timed GEMM), then times one GEMM with CUDA events. The
GEMMs stream their weight once, so the figure of merit is the weight bytes
per second against the measured copy bandwidth.

    python -m kvbm_b200.bench.gemm_bench --batch 1,8,32,64,128
"""

from __future__ import annotations

import argparse
import json

import torch

from ..ops import llama_ops

# (name, N, K): one tile (launch overhead), a 8 MiB weight, then Llama-3-8B's fused q/k/v, o,
# fused gate/up, down, lm_head
SHAPES = [("tiny", 128, 64), ("small", 1024, 4096), ("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 28672, 4096), ("down", 4096, 14336),
          ("lm_head", 128256, 4096)]


def _time(fn, iters: int, flush: torch.Tensor) -> float:
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sink = torch.empty((), dtype=flush.dtype, device=flush.device)
    best = []
    for _ in range(iters):
        torch.sum(flush, dim=0, out=sink)
        s.record()
        fn()
        e.record()
        e.synchronize()
        best.append(s.elapsed_time(e))
    best.sort()
    return best[len(best) // 2]  # median


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--batch", default="1,8,32,64,128")
    p.add_argument("--shapes", default=",".join(n for n, _, _ in SHAPES[2:]))
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--ctas", default="0", help="comma list of persistent CTA counts to try (0 = one per SM)")
    p.add_argument("--modes", default="auto", help="comma list of skinny-GEMM modes: auto, streamk, cluster")
    args = p.parse_args(argv)
    torch.cuda.set_device(0)
    flush = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
    want = set(args.shapes.split(","))
    for name, N, K in SHAPES:
        if name not in want:
            continue
        w = (torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5).to(torch.bfloat16)
        for M in (int(b) for b in args.batch.split(",")):
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            ref = x @ w.t()
            for _ in range(args.warmup):
                torch.matmul(x, w.t(), out=out)
            t_cublas = _time(lambda: torch.matmul(x, w.t(), out=out), args.iters, flush)
            wbytes = N * K * 2
            row = {"shape": name, "M": M, "N": N, "K": K, "cublas_us": round(t_cublas * 1e3, 2),
                   "cublas_gbs": round(wbytes / t_cublas / 1e6, 1)}
            runs = [(m, nc) for m in args.modes.split(",") for nc in (int(v) for v in args.ctas.split(","))
                    if nc == 0 or m == "streamk"]
            for mode, nc in runs:
                llama_ops.set_skinny_gemm_mode(mode)
                for _ in range(args.warmup):
                    llama_ops.skinny_gemm(x, w, out=out, ctas=nc)
                t = _time(lambda: llama_ops.skinny_gemm(x, w, out=out, ctas=nc), args.iters, flush)
                err = (out.float() - ref.float()).abs().max().item()
                key = f"{mode}{nc or ''}"
                row[key + "_us"] = round(t * 1e3, 2)
                row[key + "_gbs"] = round(wbytes / t / 1e6, 1)
                row[key + "_maxerr"] = round(err, 4)
            llama_ops.set_skinny_gemm_mode("auto")
            row["status"] = llama_ops.skinny_gemm_status()
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
