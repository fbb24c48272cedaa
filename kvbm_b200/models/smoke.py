"""One tiny prefill -> KV transfer -> decode step of the flagship path on cuda:0."""

from __future__ import annotations

import torch


def run_smoke() -> dict:
    from ..engine.disagg import DisaggConfig, DisaggServer
    from ..models.llama import LlamaConfig
    from ..ops import _lib

    assert torch.cuda.is_available(), "smoke() needs a CUDA GPU"
    _lib.load(build_if_missing=False)
    cfg = DisaggConfig(model=LlamaConfig.tiny(layers=2), concurrency=2, prompt_len=64, gen_len=4)
    server = DisaggServer(cfg, "colocated", 0)
    server.warmup_graphs()
    prompts = torch.randint(0, cfg.model.vocab, (cfg.concurrency, cfg.prompt_len), dtype=torch.int32).pin_memory()
    res = server.serve_wave(prompts)
    assert res.tokens is not None and tuple(res.tokens.shape) == (2, 4)
    assert res.kv_bytes == 2 * cfg.kv_bytes_per_request()
    return {"tokens": res.tokens.tolist(), "kv_bytes": res.kv_bytes, "step_ms": res.step_ms}


if __name__ == "__main__":
    print(run_smoke())
