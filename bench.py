"""Headline benchmark: intra-box disaggregated prefill/decode on Llama-3-8B.

    python bench.py --gpus N --steps K --warmup W          # this framework
    python bench.py --impl reference --gpus N ...          # the reference arm

N=1 runs prefill and decode colocated on one GPU (two instances, two KV
pools, KV moved by the same transfer kernel into the local pool); N=2,4,8
run N/2 prefill:decode pairs (1P1D, 2P2D, 4P4D), one process per GPU, ranks
[0, N/2) prefill and [N/2, N) decode, KV streamed in layer batches over
NVLink by the P2P transfer kernel. A step is one wave: ``concurrency`` requests of
``prompt_len`` uniform-random tokens per pair, prefilled one after another,
then decoded together for ``gen_len`` tokens. Weights are random-init bf16.

Reported (rank 0, one JSON line):
  value   aggregate P->D KV transfer GB/s: KV bytes moved by all pairs over
          the summed device time of the kernels that move them (max over
          prefill ranks), CUDA events around each kernel. With the default
          ``--engine tma_inline --layer-batch 8`` that kernel is the TMA
          transfer kernel, launched in the prefill stream after every 8th
          layer's KV write: bulk-async loads of the prefill pool's blocks
          into shared memory, stores straight into the decode pool's blocks
          over NVLink (layout transform / head slice / fp8 fused). With
          ``fused`` it is the RoPE + KV launch over the K/V heads, which
          stores each layer's K/V into the decode pool as it produces them;
          ``tma``/``tile`` run the copy kernel on a side stream, concurrent
          with the next GEMMs.
  ttft_p50_ms  p50 over requests of the device time from the wave start to
          the request's KV + first token landing in the decode pool.
  e2e     the same KV bytes over the whole step, timed per rank from before
          the pinned-host H2D copy of the prompts to after the D2H read of the
          generated tokens (max over ranks), through DisaggServer.serve_wave.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
from datetime import timedelta

import torch

METRIC = "P->D KV transfer GB/s + disagg p50 TTFT (Llama-3-8B, 1/2/4/8 B200, max over ranks)"


def _reference_arm(args) -> None:
    reason = ("reference cannot be installed offline: its build backend (maturin) and a Rust toolchain are "
              "absent, pip reports BackendUnavailable: No module named 'maturin'")
    if os.environ.get("RANK", "0") == "0":
        print(json.dumps({"impl": "reference", "unavailable": reason, "metric": METRIC, "n_gpus": args.gpus}))


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="kvbm", choices=["kvbm", "reference"])
    p.add_argument("--concurrency", type=int, default=32)
    p.add_argument("--prompt-len", type=int, default=8192)
    p.add_argument("--gen-len", type=int, default=256)
    p.add_argument("--engine", default="tma_inline", choices=["fused", "tma", "tile", "tma_inline", "tile_inline"],
                   help="fused: the RoPE/KV kernel stores into the decode pool; tma/tile: a copy kernel per layer "
                        "on a side stream; *_inline: that copy kernel in the prefill stream")
    p.add_argument("--max-ctas", type=int, default=0)
    p.add_argument("--layer-batch", type=int, default=8, help="copy engines: layers per transfer launch")
    p.add_argument("--layers", type=int, default=None, help="override layer count (debug only: invalid for the metric)")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--out", default=None)
    args = p.parse_args(argv)
    if args.impl == "reference":
        _reference_arm(args)
        return 0
    if args.warmup < 3 and os.environ.get("KVBM_BENCH_ALLOW_SHORT") != "1":
        print("note: warm-up below 3 steps is not a valid measurement", file=sys.stderr)

    import torch.distributed as dist

    from kvbm_b200.engine.disagg import DisaggConfig, DisaggServer
    from kvbm_b200.models.llama import LlamaConfig
    from kvbm_b200.ops import _lib
    from kvbm_b200.utils.clocks import ClockSampler

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1 and world % 2:
        raise SystemExit("multi-GPU runs need an even number of GPUs (P:D pairs)")
    torch.cuda.set_device(local)
    gloo = None
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=600))
    mcfg = LlamaConfig.llama3_8b()
    if args.layers:
        mcfg = LlamaConfig(layers=args.layers)
    cfg = DisaggConfig(model=mcfg, concurrency=args.concurrency, prompt_len=args.prompt_len, gen_len=args.gen_len,
                       engine=args.engine, max_ctas=args.max_ctas, layer_batch=args.layer_batch,
                       use_graphs=not args.no_graphs)
    half = world // 2
    if world == 1:
        role, peer = "colocated", None
    elif rank < half:
        role, peer = "prefill", rank + half
    else:
        role, peer = "decode", rank - half
    store = dist.distributed_c10d._get_default_store() if world > 1 else None
    server = DisaggServer(cfg, role, local, peer_rank=peer, group=gloo, store=store, pair_id=rank % max(1, half))
    server.connect()
    server.warmup_graphs()

    gen = torch.Generator().manual_seed(1234 + rank)

    def prompts():
        if role == "decode":
            return None
        t = torch.randint(0, mcfg.vocab, (cfg.concurrency, cfg.prompt_len), generator=gen, dtype=torch.int32)
        return t.pin_memory()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(group=gloo)
        torch.cuda.synchronize()

    # decode ranks dispatch wave k+1 before decoding wave k (prefill/decode
    # pipelining across the pair); the last timed wave dispatches nothing
    for _ in range(args.warmup):
        server.serve_wave(prompts(), more=True)
    inputs = [prompts() for _ in range(args.steps)]
    barrier()
    sampler = ClockSampler(gpus=None).start() if local == 0 else None
    launches0 = _lib.launch_count()
    results = []
    for k in range(args.steps):
        results.append(server.serve_wave(inputs[k], more=k < args.steps - 1))
    barrier()
    launches = _lib.launch_count() - launches0
    clocks = sampler.stop() if sampler else None

    mine = {
        "rank": rank, "role": role,
        "step_ms": [r.step_ms for r in results],
        "kv_ms": sum(r.kv_ms for r in results),
        "kv_bytes": sum(r.kv_bytes for r in results),
        "ttft": [t for r in results for t in r.ttft_ms],
        "decode_ms": [r.decode_ms for r in results],
        "launches": launches,
        "clocks": clocks,
    }
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, mine, group=gloo)
    else:
        allr = [mine]
    if rank == 0:
        pre = [r for r in allr if r["role"] in ("prefill", "colocated")]
        dec = [r for r in allr if r["role"] in ("decode", "colocated")]
        kv_bytes = sum(r["kv_bytes"] for r in pre)
        kv_ms = max(r["kv_ms"] for r in pre)
        value = kv_bytes / (kv_ms * 1e-3) / 1e9 if kv_ms > 0 else 0.0
        step_ms = [max(r["step_ms"][k] for r in allr) for k in range(args.steps)]
        ttft = sorted(t for r in pre for t in r["ttft"])
        itl = [d / max(1, cfg.gen_len - 1) for r in dec for d in r["decode_ms"]]
        e2e = kv_bytes / (sum(step_ms) * 1e-3) / 1e9
        clk = next((r["clocks"] for r in allr if r["clocks"]), None) or {}
        pairs = max(1, world // 2)
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(step_ms), 2),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform-random token ids, random-init weights)",
            "ttft_p50_ms": round(ttft[len(ttft) // 2], 2) if ttft else None,
            "ttft_p99_ms": round(ttft[min(len(ttft) - 1, int(len(ttft) * 0.99))], 2) if ttft else None,
            "itl_ms": round(statistics.mean(itl), 3) if itl else None,
            "kv_bytes_per_step": kv_bytes // args.steps,
            "e2e": {
                "value": round(e2e, 2), "unit": "GB/s",
                "h2d_bytes_per_step": pairs * cfg.concurrency * cfg.prompt_len * 4,
                "d2h_bytes_per_step": pairs * cfg.concurrency * cfg.gen_len * 8,
                "api": "kvbm_b200.engine.disagg.DisaggServer.serve_wave",
            },
            "gpu_launches": sum(r["launches"] for r in allr),
            "clocks": {"sm_mhz": clk.get("sm_mhz"), "sm_max_mhz": clk.get("sm_max_mhz"),
                       "reasons": clk.get("reasons", [])},
            "config": {
                "model": "Llama-3-8B" if args.layers is None else f"Llama-3-8B-{args.layers}L (debug)",
                "global_batch": cfg.concurrency * pairs,
                "seq_len": cfg.prompt_len,
                "gen_len": cfg.gen_len,
                "parallelism": "colocated" if world == 1 else f"{pairs}P{pairs}D tp1",
                "engine": cfg.engine,
                "layer_batch": cfg.layer_batch if cfg.engine != "fused" else 1,
                "prefill_attention": server.model.attention_backend,
                "l2": "inputs larger than L2 (1 GiB KV per request, 16 GB weights)",
            },
            "impl": "kvbm_b200",
        }
        print(json.dumps(line), flush=True)
        if args.out:
            with open(args.out, "w") as f:
                f.write(json.dumps(line) + "\n")
    if world > 1:
        dist.barrier(group=gloo)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
