"""Heterogeneous-TP prefill/decode through the serving engines and the connector.

Eight ranks on one box: a prefill instance with TP=4 (ranks 0-3) and two
decode instances with TP=2 (ranks 4-5 and 6-7), a Llama-architecture model
with the Llama-3-70B KV geometry (80 layers, 8 KV heads, head_dim 128;
random-init weights, each rank holding its tensor-parallel shard). Users
submit to the decode instances; their connectors send every prompt to the
prefill instance, whose four ranks each push their 2-head shard of every
layer batch into the right decode rank at the right head offset (the
``plan_push`` reshard, done by the transfer kernel's head offsets, stores
over NVLink) and publish one completion word per contributing rank in that
decode rank's host mailbox. Prompts are 4,096-32,768 tokens, length
log-uniform, token ids uniform-random.

Reported: aggregate push GB/s (bytes pushed by all prefill ranks over the
summed device time of their push launches, max over ranks), per prefill
rank GB/s, TTFT p50 (decode GPU events, submission to first token), and the
device-timed region per wave.

    torchrun --nproc-per-node 8 -m kvbm_b200.bench.tp_pd_bench
"""

from __future__ import annotations

import argparse
import json
import math
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

from ..engine.cd_plane import StorePeerDirectory, StorePrefillPlane
from ..models.llama import LlamaConfig, LlamaModel
from ..serving.engine import Request
from ..serving.pd import PdConfig, PdInstance
from ..serving.tp import create_instances


def llama3_70b(layers: int = 80) -> LlamaConfig:
    return LlamaConfig(hidden=8192, layers=layers, heads=64, kv_heads=8, head_dim=128, intermediate=28672,
                       vocab=128256, rope_theta=500000.0, max_position=33792)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--prefill-tp", type=int, default=4)
    p.add_argument("--decode-tp", type=int, default=2)
    p.add_argument("--decode-instances", type=int, default=2)
    p.add_argument("--requests", type=int, default=8, help="requests per decode instance per wave")
    p.add_argument("--min-len", type=int, default=4096)
    p.add_argument("--max-len", type=int, default=32768)
    p.add_argument("--gen", type=int, default=32)
    p.add_argument("--waves", type=int, default=2)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--layers", type=int, default=80)
    p.add_argument("--layer-batch", type=int, default=8)
    p.add_argument("--wire", default="bf16", choices=["bf16", "fp8"],
                   help="fp8: the push quantises to e4m3 (per block/layer/K-V/head scales), decode dequantises")
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    need = a.prefill_tp + a.decode_tp * a.decode_instances
    if world != need:
        raise SystemExit(f"needs {need} ranks, got {world}")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))
    ctl = dist.new_group(backend="gloo", timeout=timedelta(seconds=900))
    groups = [list(range(a.prefill_tp))]
    for d in range(a.decode_instances):
        s = a.prefill_tp + d * a.decode_tp
        groups.append(list(range(s, s + a.decode_tp)))
    tps = create_instances(groups, timeout=timedelta(seconds=900))
    tp = tps[rank]
    inst_idx = next(i for i, g in enumerate(groups) if rank in g)
    role = "prefill" if inst_idx == 0 else "decode"
    iid = 1000 + 100 * inst_idx
    mcfg = llama3_70b(a.layers)
    # one model (same seed, every TP degree slices the same full weights) on both sides of the push
    model = LlamaModel(mcfg, torch.device("cuda", local), seed=11, tp_rank=tp.rank, tp_size=tp.size,
                       tp_group=tp.nccl)
    cfg = PdConfig(model=mcfg, concurrency=a.requests, prompt_len=a.max_len, gen_len=a.gen,
                   layer_batch=a.layer_batch, decode_waves=2, prefill_requests=2, wire_dtype=a.wire)
    store = dist.distributed_c10d._get_default_store()
    plane, directory = StorePrefillPlane(store), StorePeerDirectory(store)
    inst = PdInstance(role, model, cfg, iid, plane, directory, shared=True,
                      prefill_target=1000 if role == "decode" else None, tp=tp)
    inst.warmup()
    dist.barrier(group=ctl)
    rng = np.random.default_rng(7 + inst_idx)
    total_waves = a.warmup + a.waves

    def lengths():
        return [int(round(math.exp(rng.uniform(math.log(a.min_len), math.log(a.max_len))))) for _ in range(a.requests)]

    ttft, push_ms, push_bytes = [], 0.0, 0
    t_begin = t_end = None
    served = 0
    for w in range(total_waves):
        if w == a.warmup:
            torch.cuda.synchronize()
            dist.barrier(group=ctl)
            if role == "prefill":
                inst.worker.take_push_timings()
            t_begin = torch.cuda.Event(enable_timing=True)
            t_begin.record()
        if role == "decode":
            reqs = []
            if tp.rank == 0:
                for i, n in enumerate(lengths()):
                    r = Request(f"d{inst_idx}w{w}i{i}", torch.from_numpy(
                        rng.integers(0, mcfg.vocab, n, dtype=np.int32)).pin_memory(), max_tokens=a.gen)
                    inst.engine.add_request(r)
                    reqs.append(r)
            else:
                lengths()
            # every rank of the instance steps in lockstep until rank 0 has no request left
            while True:
                busy = tp.broadcast(inst.engine.has_unfinished() if tp.rank == 0 else None)
                if not busy:
                    break
                inst.step()
            torch.cuda.synchronize()
            if tp.rank == 0 and w >= a.warmup:
                ttft += [r.arrival_event.elapsed_time(r.first_token_event) for r in reqs]
        else:
            target = (w + 1) * a.requests * a.decode_instances
            while True:
                if tp.rank == 0:
                    inst.pull(wait_s=0.0 if inst.engine.has_unfinished() else 0.01)
                state = tp.broadcast((served, inst.engine.has_unfinished() or bool(inst.engine._delayed))
                                     if tp.rank == 0 else None)
                if state[0] >= target and not state[1]:
                    break
                got = inst.step()
                if tp.rank == 0:
                    served += len(got)
            torch.cuda.synchronize()
    t_end = torch.cuda.Event(enable_timing=True)
    t_end.record()
    torch.cuda.synchronize()
    dist.barrier(group=ctl)
    if role == "prefill":
        push_ms, push_bytes = inst.worker.take_push_timings()
    mine = {"rank": rank, "role": role, "region_ms": t_begin.elapsed_time(t_end), "push_ms": push_ms,
            "push_bytes": push_bytes, "ttft": ttft, "cd": inst.leader.cd_stats if inst.leader is not None else None}
    allr = [None] * world
    dist.all_gather_object(allr, mine, group=ctl)
    if rank == 0:
        pre = [r for r in allr if r["role"] == "prefill"]
        kb = sum(r["push_bytes"] for r in pre)
        kms = max(r["push_ms"] for r in pre)
        tt = sorted(t for r in allr for t in r["ttft"])
        line = {"bench": "tp_pd", "prefill_tp": a.prefill_tp, "decode_tp": a.decode_tp,
                "decode_instances": a.decode_instances, "layers": a.layers, "kv_dtype": "bf16",
                "wire_dtype": a.wire, "note": "push GB/s counts bf16 KV bytes; with fp8 on the wire half cross NVLink",
                "push_gbps_total": round(kb / max(kms, 1e-9) / 1e6, 1),
                "push_gbps_per_prefill_rank": [round(r["push_bytes"] / max(r["push_ms"], 1e-9) / 1e6, 1) for r in pre],
                "push_bytes": kb, "waves": a.waves, "requests_per_wave": a.requests * a.decode_instances,
                "ms_per_wave": round(max(r["region_ms"] for r in allr) / a.waves, 1),
                "ttft_p50_ms": round(tt[len(tt) // 2], 1) if tt else None,
                "ttft_p99_ms": round(tt[min(len(tt) - 1, int(0.99 * len(tt)))], 1) if tt else None,
                "cd": [r["cd"] for r in allr if r["cd"] and r["role"] == "decode"]}
        print(json.dumps(line), flush=True)
        if a.out:
            with open(a.out, "a") as f:
                f.write(json.dumps(line) + "\n")
    inst.shutdown()
    dist.barrier(group=ctl)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
