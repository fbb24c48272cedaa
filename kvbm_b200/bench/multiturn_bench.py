"""Multi-turn prefix reuse with host-tier spill (one decode instance per GPU).

Every rank serves ``sessions`` chat sessions for ``turns`` turns on its own
GPU (weak scaling). All sessions share a 2,048-token system prefix; each
turn appends 256-1,024 uniform-random user tokens, is prefilled, then
decodes ``gen`` tokens, batched across a wave of sessions (as many as fit
G1 at once; a turn is several waves). G1 is a paged pool with its own
prefix cache (the serving framework's, an LRU block manager) capped at
``g1_fraction`` of the live KV, so most KV spills: the
connector offloads every completed block G1 -> G2 (pinned host) after the
forward pass and, on the next turn, onboards the G2 hits back into fresh G1
blocks with the SM gather kernel before the prefill of the new tokens.

Reported per run (max/sum over ranks): onboard GB/s (device time of the
onboard kernels), prefix hit rate split into G1 and G2 hits, TTFT p50/p99
(device time of onboard + prefill per request), tokens prefilled.

    python -m kvbm_b200.bench.multiturn_bench --sessions 64 --turns 8
    torchrun --nproc-per-node 8 -m kvbm_b200.bench.multiturn_bench
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

from ..connector.leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
from ..connector.worker import ConnectorWorker
from ..engine.leader import InstanceLeader, ParallelWorkers
from ..logical.manager import BlockManager, Tier
from ..logical.sequence import sequence_hashes
from ..models.llama import LlamaConfig, LlamaModel
from ..ops import llama_ops
from ..utils.config import KvbmConfig


def run(a, rank: int = 0) -> dict:
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    cfg = LlamaConfig.tiny(a.layers) if a.tiny else LlamaConfig(layers=a.layers)
    model = LlamaModel(cfg, "cuda", seed=rank)
    rng = np.random.default_rng(100 + rank)
    bs = 16
    vocab = cfg.vocab
    prefix = rng.integers(0, vocab, a.prefix, dtype=np.int32).tolist()
    avg_ctx = a.prefix + a.turns * ((256 + 1024) // 2 + a.gen) // 2
    live_blocks = a.sessions * math.ceil(avg_ctx * 2 / bs)
    max_req_blocks = math.ceil((a.prefix + a.turns * (1024 + a.gen)) / bs)
    g1_blocks = max(int(live_blocks * a.g1_fraction), 2 * max_req_blocks)
    # sessions resident at once: a turn is served in waves whose live KV fits G1, so
    # the prefix-cached blocks of earlier waves get evicted (spilled) by later ones
    wave = max(1, g1_blocks // max_req_blocks)
    g2_blocks = int(live_blocks * 1.2) + 64
    pool = model.allocate_pool(g1_blocks, bs)
    g1 = BlockManager(g1_blocks, bs, "lru", Tier.G1)  # the framework's own G1 prefix cache
    kcfg = KvbmConfig.load({"cache": {"host": {"num_blocks": g2_blocks}}}, env={}, system_toml=None)
    worker = ConnectorWorker(kcfg, block_size=bs, num_kv_heads=cfg.kv_heads, head_size=cfg.head_dim)
    L = cfg.layers
    worker.register_cross_layers_kv_cache(
        pool.backing.tensor(torch.bfloat16, (g1_blocks, L, 2, bs, cfg.kv_heads, cfg.head_dim)))
    leader = ConnectorLeader(InstanceLeader(BlockManager(g2_blocks, bs, "lineage", Tier.G2), ParallelWorkers([])),
                             bs)
    hist = [list(prefix) for _ in range(a.sessions)]
    ttft, onboard_ms, onboard_bytes = [], 0.0, 0
    hit_g1 = hit_g2 = total_prompt = prefilled = 0
    step = 0
    bpb = pool.config.bytes_per_block
    waves = [list(range(w, min(a.sessions, w + wave))) for w in range(0, a.sessions, wave)]
    for turn, members in ((t, m) for t in range(a.turns) for m in waves):
        held: list[list] = []
        tables, lens = [], []
        for s in members:
            hist[s] += rng.integers(0, vocab, int(rng.integers(256, 1025)), dtype=np.int32).tolist()
            toks = hist[s]
            hashes = sequence_hashes(toks, bs)
            total_prompt += len(toks)
            g1_hit = g1.match_blocks(hashes[: (len(toks) - 1) // bs])
            n1 = len(g1_hit) * bs
            rid = f"r{rank}-{turn}-{s}"
            leader.create_slot(KvbmRequest(rid, toks))
            n_ext, _ = leader.get_num_new_matched_tokens(rid, n1)
            need = math.ceil((len(toks) + a.gen) / bs) - len(g1_hit)
            fresh = g1.allocate_blocks(need)
            if fresh is None:
                raise RuntimeError("G1 too small for one request")
            ids = [b.block_id for b in g1_hit] + [b.block_id for b in fresh]
            leader.update_state_after_alloc(rid, ids, n_ext)
            step += 1
            meta = leader.build_connector_meta(SchedulerOutputLite(step, {rid: ([], [], len(toks))}))
            worker.bind_connector_metadata(meta)
            t0, t1, t2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            t0.record()
            worker.start_load_kv()
            t1.record()
            start = n1 + n_ext
            ids_t = torch.tensor(ids, dtype=torch.int32, device="cuda")
            nxt = model.prefill(torch.tensor(toks[start:], dtype=torch.int32, device="cuda"), pool, ids_t,
                                start_pos=start)
            t2.record()
            worker.wait_for_save()
            t2.synchronize()
            ttft.append(t0.elapsed_time(t2))
            if n_ext:
                onboard_ms += t0.elapsed_time(t1)
                onboard_bytes += (n_ext // bs) * bpb
            hit_g1 += n1
            hit_g2 += n_ext
            prefilled += len(toks) - start
            sending, recving = worker.get_finished({rid})
            leader.update_connector_output(sending, recving)
            leader.request_finished(rid)
            # register the prompt's full blocks in the framework's G1 cache
            nfull = len(toks) // bs
            new_full = fresh[: max(0, nfull - len(g1_hit))]
            reg = g1.register_mutable(new_full, hashes[len(g1_hit): nfull])
            held.append(g1_hit + reg + fresh[len(new_full):])
            tables.append(ids)
            lens.append(len(toks))
            hist[s].append(int(nxt))
        # batched decode of the turn (eager; contexts differ per session)
        maxb = max(len(t) for t in tables)
        table = torch.tensor([t + [t[-1]] * (maxb - len(t)) for t in tables], dtype=torch.int32, device="cuda")
        tok = torch.tensor([hist[s][-1] for s in members], dtype=torch.int64, device="cuda")
        pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
        splits = llama_ops.decode_splits(len(members), cfg.kv_heads, max(lens) + a.gen, bs)
        gen_out = []
        for _ in range(a.gen - 1):
            nt = model.decode_step(tok, pos, pool, table, pos + 1, splits)
            gen_out.append(nt)
            tok = nt
            pos = pos + 1
        if gen_out:
            gen = torch.stack(gen_out, 1).tolist()
            for k, s in enumerate(members):
                hist[s] += gen[k]
        for blocks in held:
            for b in blocks:
                b.release()
    worker.shutdown()
    ttft.sort()
    return {"rank": rank, "ttft": ttft, "onboard_ms": onboard_ms, "onboard_bytes": onboard_bytes,
            "hit_g1": hit_g1, "hit_g2": hit_g2, "total_prompt": total_prompt, "prefilled": prefilled,
            "g1_blocks": g1_blocks, "g2_blocks": g2_blocks, "live_blocks_est": live_blocks, "wave": wave}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--sessions", type=int, default=64)
    p.add_argument("--turns", type=int, default=8)
    p.add_argument("--prefix", type=int, default=2048)
    p.add_argument("--gen", type=int, default=128)
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
                "onboard_gbps": round(ob / max(oms, 1e-9) / 1e6, 1),
                "hit_rate": round(sum(r["hit_g1"] + r["hit_g2"] for r in allr) / tot, 4),
                "g1_hit_rate": round(sum(r["hit_g1"] for r in allr) / tot, 4),
                "g2_hit_rate": round(sum(r["hit_g2"] for r in allr) / tot, 4),
                "ttft_p50_ms": round(ttft[len(ttft) // 2], 2), "ttft_p99_ms": round(ttft[int(len(ttft) * 0.99)], 2),
                "prefilled_tokens": sum(r["prefilled"] for r in allr), "prompt_tokens": tot,
                "g1_blocks": allr[0]["g1_blocks"], "g2_blocks": allr[0]["g2_blocks"]}
        print(json.dumps(line), flush=True)
        if a.out:
            with open(a.out, "a") as f:
                f.write(json.dumps(line) + "\n")
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
