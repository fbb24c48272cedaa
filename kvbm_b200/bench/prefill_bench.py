"""Prefill throughput of the Llama-3-8B driver model on one GPU.

Times ``LlamaModel.prefill`` of ``--tokens`` uniform-random tokens (all 32
layers, random-init bf16 weights, K/V written into a paged pool) with CUDA
events after warm-up, and reports ms per prefill, achieved TFLOP/s (2 x
non-embedding parameters x tokens for the projections plus 2 x 2 x T^2/2 x
d_model per layer for causal attention) and the fraction of the measured
sustained cuBLAS bf16 rate in ``MEASURED_PEAKS.json`` when present.

    python -m kvbm_b200.bench.prefill_bench --tokens 8192 --iters 5
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from ..models.llama import LlamaConfig, LlamaModel


def prefill_flops(cfg: LlamaConfig, T: int) -> float:
    per_tok = 2 * (cfg.hidden * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * cfg.hidden
                   + 3 * cfg.hidden * cfg.intermediate)
    attn = 2 * 2 * (T * T / 2) * cfg.q_size  # QK^T and PV, causal half
    return cfg.layers * (per_tok * T + attn) + 2 * cfg.hidden * cfg.vocab  # + lm head of the last token


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--layers", type=int, default=None, help="debug only")
    p.add_argument("--profile", action="store_true",
                   help="bracket one extra prefill with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    a = p.parse_args(argv)
    cfg = LlamaConfig.llama3_8b() if a.layers is None else LlamaConfig(layers=a.layers)
    model = LlamaModel(cfg, "cuda", seed=0)
    page = 16
    nb = (a.tokens + page - 1) // page
    pool = model.allocate_pool(nb, page)
    ids = torch.arange(nb, dtype=torch.int32, device="cuda")
    toks = torch.randint(0, cfg.vocab, (a.tokens,), dtype=torch.int32, device="cuda")
    for _ in range(a.warmup):
        model.prefill(toks, pool, ids)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.iters)]
    for s, e in evs:
        s.record()
        model.prefill(toks, pool, ids)
        e.record()
    torch.cuda.synchronize()
    if a.profile:
        torch.cuda.profiler.start()
        model.prefill(toks, pool, ids)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    ms = sorted(s.elapsed_time(e) for s, e in evs)
    med = ms[len(ms) // 2]
    tflops = prefill_flops(cfg, a.tokens) / (med * 1e-3) / 1e12
    peak = None
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peak = json.load(f).get("bf16_tflops_sustained")
    print(json.dumps({"bench": "prefill", "model": "Llama-3-8B" if a.layers is None else f"{a.layers}L",
                      "tokens": a.tokens, "ms_median": round(med, 3), "ms_min": round(ms[0], 3),
                      "tflops": round(tflops, 1),
                      "frac_of_measured_sustained_bf16": round(tflops / peak, 3) if peak else None,
                      "attention": model.attention_backend}), flush=True)


if __name__ == "__main__":
    main()
