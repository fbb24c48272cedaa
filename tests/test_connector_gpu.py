"""Connector round trip on one GPU with the Llama harness: a cold request's
KV is offloaded G1 -> G2 by the worker, the G1 cache is wiped, and a second
request with the same prompt onboards G2 -> G1 and must produce the same
next token as the cold run (the reference's determinism test,
tests/kvbm_integration/test_determinism_agg.py)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.connector.leader import ConnectorLeader, KvbmRequest, SchedulerOutputLite
from kvbm_b200.connector.worker import ConnectorWorker
from kvbm_b200.engine.leader import InstanceLeader
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.models.llama import LlamaConfig, LlamaModel
from kvbm_b200.utils.config import KvbmConfig


@pytest.mark.parametrize("mode", ["inter", "intra"])
def test_offload_wipe_onboard_same_tokens(mode):
    cfg = LlamaConfig.tiny(layers=2)
    model = LlamaModel(cfg, "cuda", seed=3)
    NB, bs = 32, 16
    # vLLM flash-attn style per-layer tensors: [2, blocks, page, kv_heads, head_dim]
    kv = {f"model.layers.{l}.attn": torch.zeros(2, NB, bs, cfg.kv_heads, cfg.head_dim, dtype=torch.bfloat16,
                                                device="cuda") for l in range(cfg.layers)}
    kcfg = KvbmConfig.load({"cache": {"host": {"num_blocks": 64}}, "onboard": {"mode": mode}}, env={},
                           system_toml=None)
    worker = ConnectorWorker(kcfg, block_size=bs, num_kv_heads=cfg.kv_heads, head_size=cfg.head_dim)
    g1 = worker.register_kv_caches(kv, num_blocks=NB)
    assert g1.kind == "layer_separate" and not g1._block_first
    leader = ConnectorLeader(InstanceLeader.scheduler_side(BlockManager(64, bs, "lineage", Tier.G2)), bs)

    prompt = torch.randint(0, cfg.vocab, (80,), dtype=torch.int32)
    ids_a = list(range(6))
    leader.create_slot(KvbmRequest("a", prompt.tolist()))
    assert leader.get_num_new_matched_tokens("a", 0) == (0, False)
    leader.update_state_after_alloc("a", ids_a, 0)
    meta = leader.build_connector_meta(SchedulerOutputLite(1, {"a": ([], [], 80)}))
    worker.bind_connector_metadata(meta)
    worker.start_load_kv()
    tok_a = model.prefill(prompt.cuda(), g1, torch.tensor(ids_a, dtype=torch.int32, device="cuda"))
    worker.wait_for_save()
    torch.cuda.synchronize()
    sending, recving = worker.get_finished({"a"})
    assert sending == {"a"}
    wmeta = worker.build_connector_worker_meta()
    assert wmeta == {"offloaded": {1: 1}}  # step 1's copies landed: the leader may register them now
    leader.update_connector_output(sending, recving, wmeta)
    leader.request_finished("a")
    ref_blocks = g1.gather_blocks(ids_a[:4]).clone()

    for t in kv.values():
        t.zero_()

    leader.create_slot(KvbmRequest("b", prompt.tolist()))
    n, is_async = leader.get_num_new_matched_tokens("b", 0)
    assert (n, is_async) == (64, True)
    ids_b = list(range(10, 16))
    leader.update_state_after_alloc("b", ids_b, n)
    meta = leader.build_connector_meta(SchedulerOutputLite(2, {"b": ([], [], 80)}))
    worker.bind_connector_metadata(meta)
    worker.start_load_kv()
    for l in range(cfg.layers):
        worker.wait_for_layer_load(l)
    torch.cuda.synchronize()
    assert torch.equal(g1.gather_blocks(ids_b[:4]), ref_blocks)
    tok_b = model.prefill(prompt[64:].cuda(), g1, torch.tensor(ids_b, dtype=torch.int32, device="cuda"),
                          start_pos=64)
    ref = model.reference_forward(prompt.cuda())[-1]
    assert float(ref[int(tok_b)]) >= float(ref.max()) - 0.05 * float(ref.abs().max())
    assert int(tok_b) == int(tok_a)
    _, recving = worker.get_finished(set())
    assert recving == {"b"}
    worker.shutdown()
