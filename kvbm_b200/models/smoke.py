"""One tiny disaggregated serving step of the flagship path on cuda:0.

A decode instance and a prefill instance share the GPU: the decode
connector sends two prompts to the prefill instance, whose connector worker
pushes their KV into the decode pool with the TMA transfer kernel (one
launch per batch of layers) and publishes completion in the decode
instance's host mailbox; the decode engine then generates four tokens per
request with its CUDA-graph decode step.
"""

from __future__ import annotations

import torch


def run_smoke() -> dict:
    from ..engine.cd_plane import LocalPeerDirectory, LocalPrefillPlane
    from ..models.llama import LlamaConfig, LlamaModel
    from ..ops import _lib
    from ..serving.engine import Request
    from ..serving.pd import PdConfig, PdInstance

    assert torch.cuda.is_available(), "smoke() needs a CUDA GPU"
    _lib.load(build_if_missing=False)
    mcfg = LlamaConfig.tiny(layers=2)
    model = LlamaModel(mcfg, "cuda:0", seed=0)
    cfg = PdConfig(model=mcfg, concurrency=2, prompt_len=64, gen_len=4, layer_batch=1, push_engine="tma")
    plane, directory = LocalPrefillPlane(), LocalPeerDirectory()
    dec = PdInstance("decode", model, cfg, 1, plane, directory, prefill_target=2)
    pre = PdInstance("prefill", model, cfg, 2, plane, directory)
    dec.warmup()
    prompts = torch.randint(0, mcfg.vocab, (cfg.concurrency, cfg.prompt_len), dtype=torch.int32).pin_memory()
    reqs = [Request(f"smoke{i}", prompts[i], max_tokens=cfg.gen_len) for i in range(cfg.concurrency)]
    for r in reqs:
        dec.engine.add_request(r)
    for _ in range(10000):
        pre.pull()
        while pre.engine.has_unfinished():
            pre.step()
        dec.step()
        if not dec.engine.has_unfinished():
            break
    torch.cuda.synchronize()
    assert all(r.output is not None and r.output.numel() == cfg.gen_len for r in reqs)
    push_ms, push_bytes = pre.worker.take_push_timings()
    assert push_bytes == cfg.concurrency * cfg.kv_bytes_per_request(), push_bytes
    assert dec.leader.cd_stats["received"] == cfg.concurrency
    out = {"tokens": [r.output.tolist() for r in reqs], "kv_bytes": push_bytes, "push_ms": push_ms}
    dec.shutdown()
    pre.shutdown()
    return out


if __name__ == "__main__":
    print(run_smoke())
