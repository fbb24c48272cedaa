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


def test_g2_chain_to_object_store_and_fetch_back(tmp_path):
    """G4 through the connector on one GPU: the offloaded prompt blocks are uploaded to the object
    store by the worker (store op), G2 and G1 are wiped, and a second request with the same prompt
    is matched in G4, fetched into G2 and onboarded by the worker, then decodes the same token."""
    import time

    from kvbm_b200.object.store import FsObjectStore

    cfg = LlamaConfig.tiny(layers=2)
    model = LlamaModel(cfg, "cuda", seed=3)
    NB, bs = 32, 16
    kv = {f"model.layers.{l}.attn": torch.zeros(2, NB, bs, cfg.kv_heads, cfg.head_dim, dtype=torch.bfloat16,
                                                device="cuda") for l in range(cfg.layers)}
    kcfg = KvbmConfig.load({"cache": {"host": {"num_blocks": 64}},
                            "object": {"kind": "fs", "root": str(tmp_path), "lock": False}}, env={}, system_toml=None)
    worker = ConnectorWorker(kcfg, block_size=bs, num_kv_heads=cfg.kv_heads, head_size=cfg.head_dim)
    g1 = worker.register_kv_caches(kv, num_blocks=NB)
    assert worker.objects is not None
    store = FsObjectStore(str(tmp_path))
    g2 = BlockManager(64, bs, "lineage", Tier.G2)
    leader = ConnectorLeader(InstanceLeader.scheduler_side(g2), bs, objects=store)

    def run_step(step, sched):
        meta = leader.build_connector_meta(SchedulerOutputLite(step, sched))
        worker.bind_connector_metadata(meta)
        worker.start_load_kv()
        return meta

    prompt = torch.randint(0, cfg.vocab, (80,), dtype=torch.int32)
    ids_a = list(range(6))
    leader.create_slot(KvbmRequest("a", prompt.tolist()))
    assert leader.get_num_new_matched_tokens("a", 0) == (0, False)
    leader.update_state_after_alloc("a", ids_a, 0)
    run_step(1, {"a": ([], [], 80)})
    tok_a = model.prefill(prompt.cuda(), g1, torch.tensor(ids_a, dtype=torch.int32, device="cuda"))
    worker.wait_for_save()
    torch.cuda.synchronize()
    sending, recving = worker.get_finished({"a"})
    leader.update_connector_output(sending, recving, worker.build_connector_worker_meta())
    leader.request_finished("a")
    worker.clear_connector_metadata()
    ref_blocks = g1.gather_blocks(ids_a[:4]).clone()
    run_step(2, {})                               # the five registered G2 blocks chain to G4
    worker.wait_for_save()
    deadline = time.monotonic() + 30
    wmeta = None
    while time.monotonic() < deadline:
        wmeta = worker.build_connector_worker_meta()
        if wmeta and "stored" in wmeta:
            break
        time.sleep(0.01)
    assert wmeta and wmeta["stored"] == {2: 1}
    leader.update_connector_output(set(), set(), wmeta)
    worker.clear_connector_metadata()
    assert leader.engine.stats["stored_to_g4"] == 5

    g2.reset_inactive_pool()                      # G2 and G1 forget the prompt
    worker.worker.g2_layout.backing.tensor().zero_()
    for t in kv.values():
        t.zero_()
    leader.create_slot(KvbmRequest("b", prompt.tolist()))
    n, is_async = leader.get_num_new_matched_tokens("b", 0)
    assert (n, is_async) == (64, True)            # four full blocks from G4 (the last token is computed)
    ids_b = list(range(10, 16))
    leader.update_state_after_alloc("b", ids_b, n)
    meta = run_step(3, {"b": ([], [], 80)})
    for l in range(cfg.layers):
        worker.wait_for_layer_load(l)
    torch.cuda.synchronize()
    assert torch.equal(g1.gather_blocks(ids_b[:4]), ref_blocks)
    tok_b = model.prefill(prompt[64:].cuda(), g1, torch.tensor(ids_b, dtype=torch.int32, device="cuda"),
                          start_pos=64)
    assert int(tok_b) == int(tok_a)
    _, recving = worker.get_finished(set())
    assert recving == {"b"}
    leader.update_connector_output(set(), recving, None)
    assert leader.engine.stats["staged_from_g4"] == 4
    worker.shutdown()
    store.close()
