"""Facts the block manager needs from a vLLM config, and vLLM version gating.

Parity: python/kvbm/vllm/config.py:63-183 (extract_vllm_config_for_kvbm:
parallel and attention dicts, cache dtype bytes :141) and
python/kvbm/vllm/version_check.py (supported version window; the window is
widened here to the vLLM release this image ships).
"""

from __future__ import annotations

import os

SUPPORTED_VLLM = ((0, 11, 1), (0, 23, 0))  # [min, max)

_DTYPE_BYTES = {"auto": 2, "bfloat16": 2, "float16": 2, "half": 2, "fp8": 1, "fp8_e4m3": 1, "fp8_e5m2": 1,
                "float32": 4}


def cache_dtype_bytes(cache_dtype: str, model_dtype_bytes: int = 2) -> int:
    if cache_dtype in ("auto", None):
        return model_dtype_bytes
    return _DTYPE_BYTES.get(str(cache_dtype), model_dtype_bytes)


def extract_vllm_config_for_kvbm(vllm_config) -> dict:
    mc, pc, cc = vllm_config.model_config, vllm_config.parallel_config, vllm_config.cache_config
    tp = pc.tensor_parallel_size
    try:
        kv_heads = mc.get_num_kv_heads(pc)
    except Exception:  # noqa: BLE001
        kv_heads = max(1, mc.get_total_num_kv_heads() // tp)
    try:
        layers = mc.get_num_layers(pc)
    except Exception:  # noqa: BLE001
        layers = mc.hf_config.num_hidden_layers
    import torch

    model_bytes = torch.empty((), dtype=mc.dtype).element_size() if hasattr(mc, "dtype") else 2
    return {
        "block_size": cc.block_size,
        "num_layers": layers,
        "num_kv_heads": kv_heads,
        "head_size": mc.get_head_size(),
        "dtype_bytes": cache_dtype_bytes(cc.cache_dtype, model_bytes),
        "cache_dtype": str(cc.cache_dtype),
        "use_mla": bool(getattr(mc, "use_mla", False)),
        "tensor_parallel_size": tp,
        "pipeline_parallel_size": pc.pipeline_parallel_size,
        "data_parallel_size": getattr(pc, "data_parallel_size", 1),
        "data_parallel_rank": getattr(pc, "data_parallel_rank", 0),
        "rank": getattr(pc, "rank", 0),
        "max_model_len": mc.max_model_len,
    }


def kv_block_bytes(info: dict) -> int:
    outer = 1 if info.get("use_mla") else 2
    return info["num_layers"] * outer * info["block_size"] * info["num_kv_heads"] * info["head_size"] * info[
        "dtype_bytes"]


def check_vllm_version(version: str | None = None) -> None:
    if os.getenv("KVBM_SKIP_VLLM_VERSION_CHECK", "false").lower() in ("1", "true"):
        return
    if version is None:
        import vllm

        version = vllm.__version__
    parts = tuple(int("".join(c for c in p if c.isdigit()) or 0) for p in version.split(".")[:3])
    lo, hi = SUPPORTED_VLLM
    if not (lo <= parts < hi):
        raise RuntimeError(f"vLLM {version} is outside the supported range {lo}..{hi} "
                           "(set KVBM_SKIP_VLLM_VERSION_CHECK=true to override)")


def format_config_table(config: dict) -> str:
    """A fixed-width text table of a connector configuration: either sections of key/value
    pairs (``{"parallel": {...}, "attention": {...}}``) or one flat mapping (what
    :func:`extract_vllm_config_for_kvbm` returns)."""
    rule = "=" * 70
    lines = [rule, "KV block manager connector configuration", rule]
    sections = config if config and all(isinstance(v, dict) for v in config.values()) else {"settings": config}
    for name, items in sections.items():
        lines += ["", f"{str(name).replace('_', ' ').capitalize()}:", "-" * 70]
        lines += [f"  {k:30s} : {v}" for k, v in items.items()]
    lines.append(rule)
    return "\n".join(lines)
