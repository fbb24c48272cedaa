"""Headline benchmark: intra-box disaggregated prefill/decode on Llama-3-8B,
driven through the block manager's connector.

    python bench.py --gpus N --steps K --warmup W          # this framework
    python bench.py --impl reference --gpus N ...          # the reference arm

Every rank runs a serving engine (``kvbm_b200.serving``) that calls the
connector hooks (``ConnectorLeader`` / ``ConnectorWorker``) the way vLLM's v1
engine does. N=1 runs a decode instance and a prefill instance colocated on
one GPU (two KV pools; the push is a local HBM copy); N=2,4,8 run N/2
prefill:decode pairs, one process per GPU, ranks [0, N/2) prefill and
[N/2, N) decode. Users submit to the decode instances; the connector's
conditional-disaggregation policy (``always``) dispatches each prompt to the
paired prefill instance, whose connector worker pushes every batch of
``--layer-batch`` layers into the decode instance's pool over NVLink during
the prefill pass and publishes a completion word into the decode instance's
host mailbox; the decode connector reports the request received and the
engine decodes it (first step: the last prompt token, recomputed).

A step is one wave: ``concurrency`` requests of ``prompt_len`` uniform-random
tokens per pair, each generating ``gen_len`` tokens. With separate prefill
and decode GPUs the next wave is submitted once the current one has been
received (prefill of k+1 overlaps decode of k); colocated, waves run one
after another. Weights are random-init bf16.

Reported (rank 0, one JSON line):
  value   aggregate P->D KV transfer GB/s: KV bytes pushed by all prefill
          ranks over the summed device time of the push launches (CUDA events
          around each launch, max over prefill ranks).
  ms_per_step  device time of the timed region (events after the opening
          barrier and before the closing one), max over ranks, / K.
  ttft_p50_ms / p99  per request on the decode GPU: from the event recorded
          when the user submits it to the event after the decode step that
          produced its first token.
  e2e     the same KV bytes over the timed region, through the public API
          (``LLMEngine.add_request`` / ``step`` and the connector hooks),
          including every step's pinned-host upload of the prompts and the
          device-to-host read of the generated tokens.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
from datetime import timedelta

import torch

METRIC = "P->D KV transfer GB/s + disagg p50 TTFT (Llama-3-8B, 1/2/4/8 B200, max over ranks)"
HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "baseline", "_ref")


def _reference_arm(args) -> None:
    """Run the unmodified reference through its own public API, or say why it cannot run.

    The reference is a maturin/PyO3 wheel; the install is attempted here (on
    the box the bench runs on) and its own error is reported when it fails.
    """
    rank0 = os.environ.get("RANK", "0") == "0"
    reason = None
    if not os.path.isdir(os.path.join(REF_DIR, "kvbm")):
        src = "/root/reference"
        if not os.path.isdir(src):
            reason = "reference source tree not present on this box"
        elif rank0:
            try:
                r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                                    "--find-links", "/opt/wheelhouse", "--target", REF_DIR, src],
                                   capture_output=True, text=True, timeout=600)
                if r.returncode != 0:
                    tail = [ln for ln in (r.stderr or r.stdout).splitlines() if ln.strip()]
                    err = next((ln for ln in reversed(tail) if "Error" in ln or "error" in ln), tail[-1] if tail
                               else f"pip exited {r.returncode}")
                    reason = f"pip install of the reference failed on this box: {err.strip()[:300]}"
            except Exception as e:  # noqa: BLE001
                reason = f"pip install of the reference did not complete: {e}"
        else:
            reason = "reference not installed (rank 0 attempts the install)"
    if reason is None:
        try:
            sys.path.insert(0, REF_DIR)
            import kvbm  # noqa: F401  (the reference package)
            from kvbm import _core  # noqa: F401
            reason = ("the reference installed but its P->D path needs NIXL/UCX and a vLLM deployment with the "
                      "kvbm connector, which this box does not provide")
        except Exception as e:  # noqa: BLE001
            reason = f"reference package does not import: {type(e).__name__}: {e}"[:300]
    if rank0:
        print(json.dumps({"impl": "reference", "unavailable": reason, "metric": METRIC, "n_gpus": args.gpus}))


def _prompts(gen: torch.Generator, c: int, s: int, vocab: int) -> torch.Tensor:
    return torch.randint(0, vocab, (c, s), generator=gen, dtype=torch.int32).pin_memory()


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="kvbm", choices=["kvbm", "reference"])
    p.add_argument("--concurrency", type=int, default=32)
    p.add_argument("--prompt-len", type=int, default=8192)
    p.add_argument("--gen-len", type=int, default=256)
    p.add_argument("--engine", default="tma", choices=["tma", "tile"], help="push kernel")
    p.add_argument("--layer-batch", type=int, default=8, help="layers per push launch")
    p.add_argument("--layers", type=int, default=None, help="override layer count (debug only: invalid for the metric)")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--decode-stream", action="store_true",
                   help="colocated: run the decode instance on its own stream, overlapping the prefill")
    p.add_argument("--no-bulk-peer", action="store_true",
                   help="peer pushes with consumer-warp stores instead of TMA bulk stores")
    p.add_argument("--out", default=None)
    args = p.parse_args(argv)
    if args.impl == "reference":
        _reference_arm(args)
        return 0
    if args.warmup < 3 and os.environ.get("KVBM_BENCH_ALLOW_SHORT") != "1":
        print("note: warm-up below 3 steps is not a valid measurement", file=sys.stderr)

    import torch.distributed as dist

    from kvbm_b200.engine.cd_plane import (LocalPeerDirectory, LocalPrefillPlane, StorePeerDirectory,
                                           StorePrefillPlane)
    from kvbm_b200.models.llama import LlamaConfig, LlamaModel
    from kvbm_b200.ops import _lib
    from kvbm_b200.serving.engine import Request
    from kvbm_b200.serving.pd import PdConfig, PdInstance
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
    mcfg = LlamaConfig.llama3_8b() if not args.layers else LlamaConfig(layers=args.layers)
    cfg = PdConfig(model=mcfg, concurrency=args.concurrency, prompt_len=args.prompt_len, gen_len=args.gen_len,
                   layer_batch=args.layer_batch, push_engine=args.engine, use_graphs=not args.no_graphs,
                   push_bulk_peer=not args.no_bulk_peer)
    C = cfg.concurrency
    half = world // 2
    model = LlamaModel(mcfg, torch.device("cuda", local), seed=cfg.seed)
    if world == 1:
        role = "colocated"
        plane, directory = LocalPrefillPlane(), LocalPeerDirectory()
        dec = PdInstance("decode", model, cfg, 1, plane, directory, prefill_target=2)
        pre = PdInstance("prefill", model, cfg, 2, plane, directory)
    else:
        store = dist.distributed_c10d._get_default_store()
        plane, directory = StorePrefillPlane(store), StorePeerDirectory(store)
        iid = 1000 + rank
        if rank < half:
            role, dec = "prefill", None
            pre = PdInstance("prefill", model, cfg, iid, plane, directory, shared=True)
        else:
            role, pre = "decode", None
            dec = PdInstance("decode", model, cfg, iid, plane, directory, shared=True, prefill_target=1000 + rank - half)
    # colocated: the decode instance runs on its own stream, so its memory-bound decode steps overlap
    # the prefill instance's compute-bound prefill on the same GPU (the mailbox orders a request's
    # decode after its push, as across GPUs)
    dec_stream = torch.cuda.Stream() if world == 1 and args.decode_stream else None
    dec_ctx = (lambda: torch.cuda.stream(dec_stream)) if dec_stream is not None else contextlib.nullcontext
    if dec is not None:
        with dec_ctx():
            dec.warmup()
    if pre is not None:
        pre.warmup()
    torch.cuda.synchronize()

    gen = torch.Generator().manual_seed(1234 + rank)
    total = args.warmup + args.steps
    waves = [_prompts(gen, C, cfg.prompt_len, mcfg.vocab) for _ in range(total)] if dec is not None else []

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(group=gloo)
        torch.cuda.synchronize()

    submitted: dict[int, list[Request]] = {}

    def submit(k: int) -> None:
        reqs = [Request(f"r{rank}w{k}i{i}", waves[k][i], max_tokens=cfg.gen_len) for i in range(C)]
        for r in reqs:
            dec.engine.add_request(r)
        submitted[k] = reqs

    def wave_done(k: int) -> bool:
        return all(r.status.value == "finished" for r in submitted[k])

    def wave_received(k: int) -> bool:
        return all(r.status.value in ("decode", "finished") for r in submitted[k])

    served = 0

    def prefill_until(n: int) -> None:
        nonlocal served
        while served < n:
            pre.pull(wait_s=0.0 if pre.engine.has_unfinished() else 0.02)
            if pre.engine.has_unfinished() or pre.engine._delayed:
                served += len(pre.step())

    def run_wave(k: int) -> None:
        if role == "prefill":
            prefill_until((k + 1) * C)
            return
        if k not in submitted:
            with dec_ctx():
                submit(k)
        while not wave_done(k):
            if pre is not None:
                # colocated: one prefill step (one request's prompt, pushed layer batch by layer batch),
                # then one decode step, so a request starts decoding as soon as its KV has landed
                pre.pull()
                if pre.engine.has_unfinished() or pre.engine._delayed:
                    pre.step()
            with dec_ctx():
                dec.step()
            if (role == "decode" and k + 1 < total and k + 1 != args.warmup and k + 1 not in submitted
                    and wave_received(k)):
                # the next wave's prefill (on the prefill GPU) overlaps this wave's decode; not across the
                # timed edge, and not when both share one GPU (colocated: waves run one after another)
                with dec_ctx():
                    submit(k + 1)

    timed: list[Request] = []
    for k in range(args.warmup):
        run_wave(k)
    if pre is not None:
        pre.worker.take_push_timings()
    barrier()
    sampler = ClockSampler(gpus=None).start() if local == 0 else None
    launches0 = _lib.launch_count()
    t_begin = torch.cuda.Event(enable_timing=True)
    t_begin.record()
    if dec_stream is not None:
        dec_stream.wait_stream(torch.cuda.current_stream())
    for k in range(args.warmup, total):
        run_wave(k)
        if dec is not None:
            timed += submitted[k]
    t_end = torch.cuda.Event(enable_timing=True)
    if dec_stream is not None:
        torch.cuda.current_stream().wait_stream(dec_stream)
    t_end.record()
    barrier()
    launches = _lib.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    push_ms, push_bytes = pre.worker.take_push_timings() if pre is not None else (0.0, 0)
    ttft = [r.arrival_event.elapsed_time(r.first_token_event) for r in timed if r.first_token_event is not None]
    itl = [r.first_token_event.elapsed_time(r.finish_event) / max(1, r.max_tokens - 1) for r in timed
           if r.finish_event is not None and r.first_token_event is not None]
    if dec is not None:
        for r in timed:
            assert r.output is not None and r.output.numel() == cfg.gen_len, "a timed request produced no output"
    mine = {"rank": rank, "role": role, "region_ms": t_begin.elapsed_time(t_end), "push_ms": push_ms,
            "push_bytes": push_bytes, "ttft": ttft, "itl": itl, "launches": launches, "clocks": clocks,
            "cd": dec.leader.cd_stats if dec is not None else None}
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, mine, group=gloo)
    else:
        allr = [mine]
    if rank == 0:
        pre_r = [r for r in allr if r["role"] in ("prefill", "colocated")]
        kv_bytes = sum(r["push_bytes"] for r in pre_r)
        kv_ms = max(r["push_ms"] for r in pre_r)
        value = kv_bytes / (kv_ms * 1e-3) / 1e9 if kv_ms > 0 else 0.0
        region_ms = max(r["region_ms"] for r in allr)
        ms_step = region_ms / args.steps
        ttft = sorted(t for r in allr for t in r["ttft"])
        itl = [t for r in allr for t in r["itl"]]
        e2e = kv_bytes / (region_ms * 1e-3) / 1e9
        clk = next((r["clocks"] for r in allr if r["clocks"]), None) or {}
        pairs = max(1, world // 2)
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 2),
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
                "h2d_bytes_per_step": pairs * C * cfg.prompt_len * 4,
                "d2h_bytes_per_step": pairs * C * cfg.gen_len * 8,
                "api": "kvbm_b200.serving.LLMEngine.add_request/step -> ConnectorLeader/ConnectorWorker hooks "
                       "(GNMT, USAA, build_connector_meta, start_load_kv, save_kv_layer, wait_for_save, "
                       "get_finished)",
            },
            "gpu_launches": sum(r["launches"] for r in allr),
            "clocks": {"sm_mhz": clk.get("sm_mhz"), "sm_max_mhz": clk.get("sm_max_mhz"),
                       "reasons": clk.get("reasons", [])},
            "config": {
                "model": "Llama-3-8B" if args.layers is None else f"Llama-3-8B-{args.layers}L (debug)",
                "global_batch": C * pairs,
                "seq_len": cfg.prompt_len,
                "gen_len": cfg.gen_len,
                "parallelism": "colocated" if world == 1 else f"{pairs}P{pairs}D tp1",
                "colocated_streams": ("separate decode stream" if dec_stream is not None else "one stream")
                if world == 1 else None,
                "push_engine": cfg.push_engine, "push_bulk_peer": cfg.push_bulk_peer,
                "layer_batch": cfg.layer_batch,
                "cd_policy": cfg.selection,
                "prefill_attention": model.attention_backend,
                "l2": "inputs larger than L2 (1 GiB KV per request, 16 GB weights)",
            },
            "cd": next((r["cd"] for r in allr if r["cd"]), None),
            "impl": "kvbm_b200",
        }
        print(json.dumps(line), flush=True)
        if args.out:
            with open(args.out, "w") as f:
                f.write(json.dumps(line) + "\n")
    for inst in (dec, pre):
        if inst is not None:
            inst.shutdown()
    if world > 1:
        dist.barrier(group=gloo)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
