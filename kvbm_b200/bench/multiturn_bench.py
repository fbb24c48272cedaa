"""Multi-turn prefix reuse with host-tier spill (one decode instance per GPU).

Every rank runs one serving engine (``kvbm_b200.serving.LLMEngine``) with the
block manager's connector and serves ``sessions`` chat sessions for
``turns`` turns on its own GPU (weak scaling). All sessions share a
2,048-token system prefix; each turn appends 256-1,024 uniform-random user
tokens and generates ``gen`` tokens, and the next turn's prompt is the whole
conversation so far. The engine keeps its own G1 prefix cache (finished
prompts' full blocks stay registered in an LRU block manager) capped at
``g1_fraction`` of the live KV, so most KV spills: the connector offloads
every completed prompt block G1 -> G2 (pinned host) after the forward pass
(registered in G2 once the copy is reported done) and, when a later turn's
prompt misses G1, onboards the G2 hits back into fresh G1 blocks with the
SM gather kernel before the new tokens are prefilled. All of a turn's
requests are submitted at once; the engine admits them as G1 allows and
decodes up to 32 at a time.

Reported per run (sum / max over ranks): onboard GB/s (device time of the
onboard transfers, CUDA events on the onboard stream), prefix hit rate split
into G1 and G2 hits, TTFT p50/p99 (per request on its GPU: the event at
submission to the event after the step that produced its first token),
tokens prefilled.

    python -m kvbm_b200.bench.multiturn_bench --sessions 64 --turns 8
    torchrun --nproc-per-node 8 -m kvbm_b200.bench.multiturn_bench     # 512 sessions x 8 turns
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

from ..connector.leader import ConnectorLeader
from ..connector.worker import ConnectorWorker
from ..engine.leader import InstanceLeader
from ..logical.manager import BlockManager, Tier
from ..models.llama import LlamaConfig, LlamaModel
from ..serving.engine import EngineConfig, LLMEngine, Request
from ..utils.config import KvbmConfig


def run(a, rank: int = 0) -> dict:
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    cfg = LlamaConfig.tiny(a.layers) if a.tiny else LlamaConfig(layers=a.layers)
    model = LlamaModel(cfg, torch.device("cuda", local), seed=rank)
    rng = np.random.default_rng(100 + rank)
    bs = 16
    prefix = rng.integers(0, cfg.vocab, a.prefix, dtype=np.int32)
    max_ctx = a.prefix + a.turns * (1024 + a.gen)
    # live KV at the end of the run (every session's whole conversation)
    mean_ctx_end = a.prefix + a.turns * ((256 + 1024) // 2 + a.gen)
    live_blocks = a.sessions * math.ceil(mean_ctx_end / bs)
    max_req_blocks = math.ceil(max_ctx / bs)
    g1_blocks = max(int(live_blocks * a.g1_fraction), 2 * max_req_blocks) + 1
    g2_blocks = int(live_blocks * 1.2) + 64
    kcfg = KvbmConfig.load({"cache": {"host": {"num_blocks": g2_blocks}}}, env={}, system_toml=None)
    leader = ConnectorLeader(InstanceLeader.scheduler_side(BlockManager(g2_blocks, bs, "lineage", Tier.G2)),
                             bs)
    worker = ConnectorWorker(kcfg, device=local, block_size=bs)
    eng = LLMEngine(model, EngineConfig(num_gpu_blocks=g1_blocks, block_size=bs, max_num_seqs=a.batch,
                                        max_num_batched_tokens=8192, max_model_len=max_ctx + a.gen,
                                        max_tokens=a.gen, prefix_caching=True), leader, worker)
    worker.register_layout(eng.pool)
    worker.onboard_timing = True
    eng.warmup()
    hist = [prefix.copy() for _ in range(a.sessions)]
    ttft: list[float] = []
    onboard_ms = 0.0
    onboard_bytes = 0
    for turn in range(a.turns):
        reqs = []
        for s in range(a.sessions):
            hist[s] = np.concatenate([hist[s], rng.integers(0, cfg.vocab, int(rng.integers(256, 1025)),
                                                            dtype=np.int32)])
            r = Request(f"r{rank}-t{turn}-s{s}", torch.from_numpy(hist[s].copy()).pin_memory(), max_tokens=a.gen)
            eng.add_request(r)
            reqs.append(r)
        while eng.has_unfinished() or eng._delayed:
            eng.step()
        torch.cuda.synchronize()
        for s, r in enumerate(reqs):
            hist[s] = np.concatenate([hist[s], r.output.numpy().astype(np.int32)])
            ttft.append(r.arrival_event.elapsed_time(r.first_token_event))
        ms, nb = worker.take_onboard_timings()
        onboard_ms += ms
        onboard_bytes += nb
    st = dict(eng.stats)
    worker.shutdown()
    ttft.sort()
    return {"rank": rank, "ttft": ttft, "onboard_ms": onboard_ms, "onboard_bytes": onboard_bytes,
            "hit_g1": st["g1_hit_tokens"], "hit_g2": st["external_tokens"], "total_prompt": st["prompt_tokens"],
            "prefilled": st["prefill_tokens"], "decode_steps": st["decode_steps"], "g1_blocks": g1_blocks,
            "g2_blocks": g2_blocks, "live_blocks_est": live_blocks}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--sessions", type=int, default=64, help="sessions per GPU (8 GPUs x 64 = 512)")
    p.add_argument("--turns", type=int, default=8)
    p.add_argument("--prefix", type=int, default=2048)
    p.add_argument("--gen", type=int, default=128)
    p.add_argument("--batch", type=int, default=32, help="decode batch slots")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--g1-fraction", type=float, default=0.3)
    p.add_argument("--tiny", action="store_true")
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=1800))
    res = run(a, rank)
    allr = [res]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, res)
    if rank == 0:
        ttft = sorted(t for r in allr for t in r["ttft"])
        ob = sum(r["onboard_bytes"] for r in allr)
        oms = max(r["onboard_ms"] for r in allr)
        tot = sum(r["total_prompt"] for r in allr)
        line = {"bench": "multiturn_spill", "gpus": world, "sessions_per_gpu": a.sessions, "turns": a.turns,
                "sessions_total": a.sessions * world,
                "onboard_gbps_per_gpu": round(sum(r["onboard_bytes"] / max(r["onboard_ms"], 1e-9) / 1e6
                                                  for r in allr) / world, 1),
                "onboard_gbps_total": round(ob / max(oms, 1e-9) / 1e6, 1),
                "onboard_bytes": ob,
                "hit_rate": round(sum(r["hit_g1"] + r["hit_g2"] for r in allr) / tot, 4),
                "g1_hit_rate": round(sum(r["hit_g1"] for r in allr) / tot, 4),
                "g2_hit_rate": round(sum(r["hit_g2"] for r in allr) / tot, 4),
                "ttft_p50_ms": round(ttft[len(ttft) // 2], 2), "ttft_p99_ms": round(ttft[int(len(ttft) * 0.99)], 2),
                "prefilled_tokens": sum(r["prefilled"] for r in allr), "prompt_tokens": tot,
                "g1_blocks": allr[0]["g1_blocks"], "g2_blocks": allr[0]["g2_blocks"],
                "g1_fraction_of_live": round(allr[0]["g1_blocks"] / allr[0]["live_blocks_est"], 3),
                "ttft_p50_p99_ms_per_rank": [[round(r["ttft"][len(r["ttft"]) // 2], 1),
                                              round(r["ttft"][int(len(r["ttft"]) * 0.99)], 1)] for r in allr]}
        print(json.dumps(line), flush=True)
        if a.out:
            with open(a.out, "a") as f:
                f.write(json.dumps(line) + "\n")
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
