"""A real vLLM engine with the block manager's connector on one B200.

vLLM 0.22 serves a random-init Llama-architecture model (``load_format=
"dummy"``, token-id prompts, no tokenizer) with ``KvbmConnector`` as its KV
connector. Greedy outputs must be identical before and after the prefix
cache is reset, and the second pass must be served from G2: the connector's
GNMT reports matched tokens, its workers onboard them (the reference's
determinism test, tests/kvbm_integration/test_determinism_agg.py:156-191).
"""

import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _tiny_llama_dir(path):
    cfg = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 1024,
        "intermediate_size": 2048, "num_hidden_layers": 2, "num_attention_heads": 8, "num_key_value_heads": 2,
        "head_dim": 128, "vocab_size": 2048, "max_position_embeddings": 4096, "rms_norm_eps": 1e-5,
        "rope_theta": 500000.0, "torch_dtype": "bfloat16", "tie_word_embeddings": False, "bos_token_id": 1,
        "eos_token_id": 2, "hidden_act": "silu",
    }
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    return path


def _connector(llm):
    """The scheduler-side KvbmConnector of an in-process engine core (None if not reachable)."""
    core = getattr(llm.llm_engine, "engine_core", None)
    core = getattr(core, "engine_core", core)
    sched = getattr(core, "scheduler", None)
    return getattr(sched, "connector", None)


def test_vllm_engine_outputs_identical_after_prefix_cache_reset(tmp_path, monkeypatch):
    pytest.importorskip("vllm")
    monkeypatch.setenv("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    from vllm import LLM, SamplingParams
    from vllm.config import KVTransferConfig
    from vllm.inputs import TokensPrompt

    import gc

    gc.collect()
    torch.cuda.empty_cache()  # vLLM sizes its cache from the memory free now
    model_dir = _tiny_llama_dir(str(tmp_path / "tiny-llama"))
    ktc = KVTransferConfig(kv_connector="KvbmConnector", kv_connector_module_path="kvbm_b200.connector.vllm_connector",
                           kv_role="kv_both",
                           kv_connector_extra_config={"leader": {"cache": {"host": {"num_blocks": 256}}},
                                                      "worker": {"cache": {"host": {"num_blocks": 256}}}})
    llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
              gpu_memory_utilization=0.3, max_model_len=1024, block_size=16, dtype="bfloat16",
              enable_prefix_caching=True, kv_transfer_config=ktc, seed=0)
    g = torch.Generator().manual_seed(5)
    prompts = [TokensPrompt(prompt_token_ids=torch.randint(3, 2000, (n,), generator=g).tolist())
               for n in (200, 333, 97)]
    sp = SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True, detokenize=False)
    first = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    # the offloads of the finished requests still hold their G1 blocks until the workers report them
    # (finished_sending) in later engine steps: step the idle engine until the cache can be reset
    for _ in range(200):
        if llm.reset_prefix_cache():
            break
        llm.llm_engine.step()
    else:
        raise AssertionError("prefix cache never became resettable")
    second = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert [list(x) for x in first] == [list(x) for x in second]
    conn = _connector(llm)
    if conn is not None and getattr(conn, "_leader", None) is not None:
        lead = conn._leader
        # the second pass found the prompts' full blocks in G2 (all but the last prompt token's block)
        assert lead.leader.stats["g2_hits"] >= sum((len(p["prompt_token_ids"]) - 1) // 16 for p in prompts)
        # ... and its workers onboarded them into vLLM's G1 blocks
        assert lead.tier_stats["onboarded_blocks"] >= sum((len(p["prompt_token_ids"]) - 1) // 16 for p in prompts)
        assert lead.tier_stats["offload_ops"] > 0
