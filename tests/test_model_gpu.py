"""Llama harness + disaggregated serving path on one GPU."""

import pytest
import torch

pytestmark = pytest.mark.gpu

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


@pytest.mark.parametrize("engine", ["tma", "tile"])
def test_serving_waves_with_graphs(engine):
    """Two waves through the disaggregated serving path (colocated), decode steps as CUDA graphs."""
    from kvbm_b200.engine.cd_plane import LocalPeerDirectory, LocalPrefillPlane
    from kvbm_b200.serving.engine import Request
    from kvbm_b200.serving.pd import PdConfig, PdInstance

    mcfg = LlamaConfig.tiny(layers=2)
    model = LlamaModel(mcfg, "cuda", seed=2)
    cfg = PdConfig(model=mcfg, concurrency=3, prompt_len=80, gen_len=5, push_engine=engine, layer_batch=2)
    plane, directory = LocalPrefillPlane(), LocalPeerDirectory()
    dec = PdInstance("decode", model, cfg, 1, plane, directory, prefill_target=2)
    pre = PdInstance("prefill", model, cfg, 2, plane, directory)
    dec.warmup()
    assert dec.engine.batch.graph is not None
    prompts = torch.randint(0, mcfg.vocab, (3, 80), dtype=torch.int32).pin_memory()
    outs = []
    for wave in range(2):
        reqs = [Request(f"w{wave}r{i}", prompts[i], max_tokens=5) for i in range(3)]
        for r in reqs:
            dec.engine.add_request(r)
        while dec.engine.has_unfinished():
            pre.pull()
            while pre.engine.has_unfinished():
                pre.step()
            dec.step()
        torch.cuda.synchronize()
        outs.append(torch.stack([r.output for r in reqs]))
        assert all(r.arrival_event.elapsed_time(r.first_token_event) > 0 for r in reqs)
    for r in range(3):
        _check_greedy(model, prompts[r].tolist() + outs[0][r].tolist(), 80)
    # the second wave reuses the graph, the pools and the mailbox slots
    assert torch.equal(outs[0], outs[1])
    assert pre.worker.take_push_timings()[1] == 6 * cfg.kv_bytes_per_request()
    dec.shutdown()
    pre.shutdown()


def test_smoke_entry():
    from kvbm_b200.models.smoke import run_smoke

    out = run_smoke()
    assert out["kv_bytes"] > 0
