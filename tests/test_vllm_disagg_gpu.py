"""Conditional disaggregation between two real vLLM engines, joined by the block manager's connector.

A prefill engine and a decode engine (vLLM 0.22, random-init Llama-architecture model,
``load_format="dummy"``, token-id prompts) run in two processes on one GPU, each with
``KvbmConnector`` configured for its disaggregation role. The decode engine's connector sends
every prompt to the prefill engine over the on-node plane (a shared directory), the prefill
engine's connector pushes the prompt's KV from its own vLLM KV cache into the decode engine's
vLLM KV cache (mapped through PyTorch's CUDA IPC records of the decode engine's tensors) during
the prefill forward pass, and the decode engine's connector reports the request received once
the completion word lands. Checked:

* every request went remote and landed (no load error, no recompute);
* the pushed KV is byte-identical on both sides (per-block checksums of the prefill engine's
  source blocks against the decode engine's destination blocks);
* greedy outputs are deterministic under disaggregation: the same prompts served twice through
  the remote path give the same tokens (the reference's disaggregated determinism test,
  tests/kvbm_integration/test_determinism_disagg.py).

The two engines only meet through files, a shared-memory mailbox and the mapped pool; no GPU
wait spans the two processes (the decode side polls its mailbox on the host).
"""

import json
import os
import subprocess
import sys
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.abspath(__file__)
PROMPT_LENS = (211, 333, 97, 160)
GEN = 8


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


def _engine(model_dir, disagg):
    from vllm import LLM
    from vllm.config import KVTransferConfig

    ktc = KVTransferConfig(kv_connector="KvbmConnector", kv_connector_module_path="kvbm_b200.connector.vllm_connector",
                           kv_role="kv_both", kv_connector_extra_config={"disagg": disagg})
    return LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
               gpu_memory_utilization=0.15, max_model_len=1024, block_size=16, dtype="bfloat16",
               enable_prefix_caching=False, kv_transfer_config=ktc, seed=0)


def _worker():
    from vllm.distributed.kv_transfer import get_kv_transfer_group

    return get_kv_transfer_group()._worker


def _scheduler_connector(llm):
    core = getattr(llm.llm_engine, "engine_core", None)
    core = getattr(core, "engine_core", core)
    return getattr(getattr(core, "scheduler", None), "connector", None)


def _checksums(worker, ids):
    from kvbm_b200.physical.verify import checksum_blocks

    torch.cuda.synchronize()
    return dict(zip([int(i) for i in ids], checksum_blocks(worker.g1, ids)))


def _prefill_main(model_dir, root, iid, out_path):
    """Serve dispatches from the plane until the stop file appears; report what was pushed."""
    from vllm import SamplingParams
    from vllm.inputs import TokensPrompt

    from kvbm_b200.connector.leader import REMOTE_DECODE_KEY
    from kvbm_b200.engine.cd_plane import FilePrefillPlane

    llm = _engine(model_dir, {"role": "prefill", "instance_id": iid, "directory": f"file://{root}"})
    w = _worker()
    w.transfer_log = []
    plane = FilePrefillPlane(root)
    open(os.path.join(root, "prefill.ready"), "w").close()
    pushed = {}  # decode block id -> checksum of the prefill block stored there (last writer wins)
    stop = os.path.join(root, "stop")
    while not os.path.exists(stop):
        got = plane.wait(iid, 0.2)
        if not got:
            continue
        prompts, sps = [], []
        for d in got:
            params = dict(d["params"])
            params[REMOTE_DECODE_KEY] = d["decode"]
            prompts.append(TokensPrompt(prompt_token_ids=[int(t) for t in d["tokens"]]))
            sps.append(SamplingParams(max_tokens=1, temperature=0.0, detokenize=False,
                                      extra_args={"kv_transfer_params": params}))
        llm.generate(prompts, sps, use_tqdm=False)
        log, w.transfer_log = w.transfer_log, []
        for kind, _rid, _peer, src, dst in (e for e in log if e[0] == "push"):
            sums = _checksums(w, src)
            pushed.update({int(d): sums[int(s)] for s, d in zip(src, dst)})
        with open(out_path, "w") as f:
            json.dump({"pushed": {str(k): v for k, v in pushed.items()}}, f)


def _decode_main(model_dir, root, iid, prefill_iid, out_path):
    from vllm import SamplingParams
    from vllm.inputs import TokensPrompt

    llm = _engine(model_dir, {"role": "decode", "instance_id": iid, "prefill_instance": prefill_iid,
                              "selection": "always", "directory": f"file://{root}", "mailbox_slots": 16,
                              "recv_timeout_s": 120})
    w = _worker()
    w.transfer_log = []
    g = torch.Generator().manual_seed(5)
    prompts = [TokensPrompt(prompt_token_ids=torch.randint(3, 2000, (n,), generator=g).tolist()) for n in PROMPT_LENS]
    sp = SamplingParams(max_tokens=GEN, temperature=0.0, ignore_eos=True, detokenize=False)
    runs, received = [], []
    for _ in range(2):
        outs = llm.generate(prompts, sp, use_tqdm=False)
        runs.append([list(o.outputs[0].token_ids) for o in outs])
        log, w.transfer_log = w.transfer_log, []
        # blocks wholly inside the pushed positions [0, len - 1): the decode engine recomputes the last
        # prompt token and writes generated tokens after it, so later blocks legitimately differ
        recv = [e for e in log if e[0] == "recv"]
        sums = {}
        for _kind, _rid, ids in recv:
            sums.update(_checksums(w, ids))
        received.append({"recv": [list(map(int, ids)) for _k, _r, ids in recv], "sums": sums})
    conn = _scheduler_connector(llm)
    cd = dict(conn._leader.cd_stats) if conn is not None and getattr(conn, "_leader", None) is not None else None
    with open(out_path, "w") as f:
        json.dump({"runs": runs, "received": [{"recv": r["recv"], "sums": {str(k): v for k, v in r["sums"].items()}}
                                              for r in received], "cd": cd, "lens": list(PROMPT_LENS)}, f)


def _run_pair(tmp_path, prefill_gpu: str, decode_gpu: str):
    """Start the prefill engine on ``prefill_gpu`` and the decode engine on ``decode_gpu`` (each process
    sees only its own GPU) and check the disaggregated run."""
    import gc

    gc.collect()
    torch.cuda.empty_cache()  # earlier tests in this process must not hold the memory the engines ask for
    model_dir = _tiny_llama_dir(str(tmp_path / "tiny-llama"))
    root = str(tmp_path / "plane")
    os.makedirs(root)
    base = int.from_bytes(os.urandom(2), "little") * 16 + 4096
    pre_iid, dec_iid = base + 1, base + 2
    repo = os.path.dirname(os.path.dirname(HERE))
    env = {**os.environ, "VLLM_ENABLE_V1_MULTIPROCESSING": "0",
           "PYTHONPATH": os.pathsep.join([repo] + [p for p in [os.environ.get("PYTHONPATH")] if p])}
    pre_env, dec_env = {**env, "CUDA_VISIBLE_DEVICES": prefill_gpu}, {**env, "CUDA_VISIBLE_DEVICES": decode_gpu}
    pre_out, dec_out = str(tmp_path / "prefill.json"), str(tmp_path / "decode.json")
    pre = subprocess.Popen([sys.executable, HERE, "prefill", model_dir, root, str(pre_iid), pre_out], env=pre_env)
    dec = None
    try:
        deadline = time.monotonic() + 300
        # on one GPU the engines start one after the other (each sizes its cache from the free memory);
        # on two GPUs the decode engine starts at once and its dispatches wait in the plane
        while prefill_gpu == decode_gpu and not os.path.exists(os.path.join(root, "prefill.ready")):
            assert pre.poll() is None, f"prefill engine exited with {pre.returncode}"
            assert time.monotonic() < deadline, "prefill engine did not start"
            time.sleep(0.5)
        dec = subprocess.Popen([sys.executable, HERE, "decode", model_dir, root, str(dec_iid), str(pre_iid), dec_out],
                               env=dec_env)
        assert dec.wait(timeout=600) == 0, "decode engine failed"
    finally:
        open(os.path.join(root, "stop"), "w").close()
        for p in (dec, pre):
            if p is None:
                continue
            try:
                p.wait(timeout=120)
            except subprocess.TimeoutExpired:
                p.kill()
                p.wait()
    assert pre.returncode == 0, "prefill engine failed"
    with open(dec_out) as f:
        d = json.load(f)
    with open(pre_out) as f:
        pushed = {int(k): v for k, v in json.load(f)["pushed"].items()}
    n = len(PROMPT_LENS)
    assert d["cd"] is not None
    assert d["cd"]["remote"] == d["cd"]["dispatched"] == d["cd"]["received"] == 2 * n, d["cd"]
    assert d["cd"]["failed"] == 0
    # deterministic greedy outputs through the remote path, full length
    assert d["runs"][0] == d["runs"][1]
    assert all(len(t) == GEN for t in d["runs"][0])
    # the KV that landed is the KV the prefill engine computed, byte for byte (last run's blocks)
    last = d["received"][1]
    sums = {int(k): v for k, v in last["sums"].items()}
    checked = 0
    by_blocks = {-(-p // 16): p for p in PROMPT_LENS}  # the prompts' block counts differ
    assert len(last["recv"]) == n
    for ids in last["recv"]:
        plen = by_blocks[len(ids)]  # nothing was provided locally: every prompt block is received
        for i in ids[: (plen - 1) // 16]:
            assert i in pushed, f"decode block {i} was never pushed"
            assert sums[i] == pushed[i], f"decode block {i}: checksum differs from the prefill block pushed there"
            checked += 1
    assert checked >= sum((p - 1) // 16 for p in PROMPT_LENS)


def _visible_gpus() -> list[str]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    ids = [g for g in vis.split(",") if g] if vis else [str(i) for i in range(torch.cuda.device_count())]
    return ids


def test_vllm_engines_disaggregated_through_the_connector(tmp_path):
    pytest.importorskip("vllm")
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    g = _visible_gpus()[0]
    _run_pair(tmp_path, g, g)


@pytest.mark.multigpu
def test_vllm_engines_on_two_gpus_push_over_nvlink(tmp_path):
    """The same with each engine on its own GPU, each process seeing only that GPU: the prefill
    engine's worker maps the decode engine's KV cache from the other GPU and pushes over NVLink."""
    pytest.importorskip("vllm")
    gpus = _visible_gpus() if torch.cuda.is_available() else []
    if len(gpus) < 2:
        pytest.skip("needs two GPUs")
    _run_pair(tmp_path, gpus[1], gpus[0])


if __name__ == "__main__":
    if sys.argv[1] == "prefill":
        _prefill_main(sys.argv[2], sys.argv[3], int(sys.argv[4]), sys.argv[5])
    else:
        _decode_main(sys.argv[2], sys.argv[3], int(sys.argv[4]), int(sys.argv[5]), sys.argv[6])
