"""Llama harness + disaggregated serving path on one GPU."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.engine.disagg import DisaggConfig, DisaggServer
from kvbm_b200.models.llama import LlamaConfig, LlamaModel


def _check_greedy(model, seq, first_gen_pos, tol=0.05):
    """Every generated token must be (near-)argmax of the fp32 reference."""
    ref = model.reference_forward(torch.tensor(seq, device=model.device))
    for pos in range(first_gen_pos - 1, len(seq) - 1):
        row = ref[pos]
        assert float(row[seq[pos + 1]]) >= float(row.max()) - tol * float(row.abs().max()), pos


@pytest.mark.parametrize("gemm", ["cublas", "tc"])
def test_prefill_decode_matches_reference(gemm):
    torch.manual_seed(0)
    cfg = LlamaConfig.tiny(layers=2)
    model = LlamaModel(cfg, "cuda", seed=1)
    model.decode_gemm = gemm
    pool = model.allocate_pool(16)
    T = 45
    prompt = torch.randint(0, cfg.vocab, (T,), device="cuda", dtype=torch.int32)
    ids = torch.tensor([3, 7, 1, 12, 5], dtype=torch.int32, device="cuda")
    tok = model.prefill(prompt, pool, ids)
    seq = prompt.tolist() + [int(tok)]
    table = ids.view(1, -1)
    for step in range(6):
        pos = torch.tensor([T + step], dtype=torch.int32, device="cuda")
        nxt = model.decode_step(torch.tensor([seq[-1]], device="cuda"), pos, pool, table, pos + 1, splits=2)
        seq.append(int(nxt))
    _check_greedy(model, seq, T)


@pytest.mark.parametrize("engine", ["fused", "tma", "tma_inline"])
def test_colocated_wave_and_graphs(engine):
    cfg = DisaggConfig(model=LlamaConfig.tiny(layers=2), concurrency=3, prompt_len=80, gen_len=5, engine=engine)
    server = DisaggServer(cfg, "colocated", 0)
    server.warmup_graphs()
    prompts = torch.randint(0, cfg.model.vocab, (3, 80), dtype=torch.int32).pin_memory()
    res = server.serve_wave(prompts)
    assert res.tokens.shape == (3, 5)
    assert res.kv_bytes == 3 * cfg.kv_bytes_per_request()
    assert len(res.ttft_ms) == 3 and all(t > 0 for t in res.ttft_ms)
    # the decode pool holds exactly the prefill KV: check every request's greedy tokens
    for r in range(3):
        seq = prompts[r].tolist() + res.tokens[r].tolist()
        _check_greedy(server.model, seq, 80)
    # a second wave reuses the graph and the pools
    res2 = server.serve_wave(prompts)
    assert torch.equal(res2.tokens, res.tokens)


def test_smoke_entry():
    from kvbm_b200.models.smoke import run_smoke

    out = run_smoke()
    assert out["kv_bytes"] > 0
