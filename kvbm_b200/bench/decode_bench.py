"""Decode-step microbenchmark: batch ``B`` of Llama-3-8B requests with a
``ctx``-token paged KV context, one decode step per iteration (CUDA graph
or eager). Prints ms/step and the share spent in paged decode attention
(timed separately on the same inputs).

    python -m kvbm_b200.bench.decode_bench --batch 32 --ctx 8448
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from ..models.llama import LlamaConfig, LlamaModel
from ..ops import llama_ops


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--ctx", type=int, default=8448)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--eager", action="store_true")
    p.add_argument("--splits", type=int, default=0)
    p.add_argument("--gemm", default="cublas", choices=["cublas", "tc"],
                   help="decode projections: cuBLAS or the tcgen05 skinny GEMM")
    p.add_argument("--no-pdl", action="store_true", help="launch the skinny GEMM without programmatic dependent launch")
    p.add_argument("--profile", action="store_true",
                   help="bracket one extra eager step with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    args = p.parse_args(argv)
    torch.cuda.set_device(0)
    cfg = LlamaConfig(layers=args.layers)
    model = LlamaModel(cfg, "cuda")
    model.decode_gemm = args.gemm
    llama_ops.set_skinny_gemm_pdl(not args.no_pdl)
    page = 16
    bpr = math.ceil((args.ctx + 1) / page)
    pool = model.allocate_pool(args.batch * bpr + 1, page)
    for l in range(cfg.layers):
        pool.layer_view(l).normal_(0, 1)
    B = args.batch
    table = torch.arange(B * bpr, dtype=torch.int32, device="cuda").view(B, bpr)
    tok = torch.randint(0, cfg.vocab, (B,), device="cuda")
    pos = torch.full((B,), args.ctx, dtype=torch.int32, device="cuda")
    seq = pos + 1
    splits = args.splits or llama_ops.decode_splits(B, cfg.kv_heads, args.ctx + 1, page)

    def step():
        nxt = model.decode_step(tok, pos, pool, table, seq, splits)
        tok.copy_(nxt)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    g = None
    if not args.eager:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        g.replay() if g is not None else step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    if args.profile:
        torch.cuda.profiler.start()
        step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    # attention alone, all layers, same inputs
    q = torch.randn(B, cfg.heads, cfg.head_dim, device="cuda", dtype=torch.bfloat16)
    scratch = model.decode_scratch(B, splits)
    counters = model.decode_counters(B)
    out = torch.empty_like(q)

    def attn():
        for l in range(cfg.layers):
            kb, vb = model.kv_bases(pool, l)
            llama_ops.paged_decode_attn(q, kb, vb, pool.block_stride, pool.token_stride, pool.head_stride, page,
                                        table, seq, cfg.kv_heads, model.scale, splits, scratch=scratch, out=out,
                                        counters=counters)
    for _ in range(2):
        attn()
    torch.cuda.synchronize()
    s.record()
    for _ in range(args.steps):
        attn()
    e.record()
    torch.cuda.synchronize()
    attn_ms = s.elapsed_time(e) / args.steps
    kv_bytes = cfg.layers * B * (args.ctx + 1) * 2 * cfg.kv_heads * cfg.head_dim * 2
    print(json.dumps({"batch": B, "ctx": args.ctx, "splits": splits, "gemm": args.gemm, "pdl": not args.no_pdl, "ms_per_step": round(ms, 3),
                      "attn_ms": round(attn_ms, 3), "attn_gbps": round(kv_bytes / attn_ms / 1e6, 1),
                      "weights_gb": round(cfg.num_params() * 2 / 1e9, 2)}))


if __name__ == "__main__":
    main()
