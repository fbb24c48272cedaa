"""``kvbm.vllm.config``: the vLLM facts the connector sizes its pools from, and their table.

``extract_vllm_config_for_kvbm`` here returns a ``KvbmVllmConfig`` with the reference's
``parallel`` and ``attention`` sections (and prints the table on rank 0 when ``log_config``);
``kvbm_b200.connector.config.extract_vllm_config_for_kvbm`` is the flat form the connector uses.
"""

from kvbm_b200._core import KvbmVllmConfig
from kvbm_b200.connector.config import extract_vllm_config_for_kvbm as _flat
from kvbm_b200.connector.config import format_config_table, kv_block_bytes  # noqa: F401


def _kv_cache_layout(vllm_config) -> str:
    try:
        from vllm.config import set_current_vllm_config
        from vllm.distributed.kv_transfer.kv_connector.utils import get_kv_cache_layout

        with set_current_vllm_config(vllm_config):
            return str(get_kv_cache_layout())
    except Exception:  # noqa: BLE001 - the layout is informative; a config without it reads NHD
        return "NHD"


def extract_vllm_config_for_kvbm(vllm_config, log_config: bool = True) -> KvbmVllmConfig:
    flat = _flat(vllm_config)
    pc, cc, mc = vllm_config.parallel_config, vllm_config.cache_config, vllm_config.model_config
    parallel = {"world_size": getattr(pc, "world_size", 1), "rank": getattr(pc, "rank", 0),
                "tensor_parallel_size": pc.tensor_parallel_size, "pipeline_parallel_size": pc.pipeline_parallel_size,
                "data_parallel_size": getattr(pc, "data_parallel_size", 1),
                "data_parallel_rank": getattr(pc, "data_parallel_rank", 0),
                "backend": getattr(pc, "data_parallel_backend", None)}
    try:
        heads = mc.get_total_num_kv_heads()
    except Exception:  # noqa: BLE001
        heads = flat["num_kv_heads"] * max(1, pc.tensor_parallel_size)
    attention = {"block_size": cc.block_size, "num_gpu_blocks": getattr(cc, "num_gpu_blocks", None) or 0,
                 "num_cpu_blocks": getattr(cc, "num_cpu_blocks", None) or 0,
                 "cache_dtype_bytes": flat["dtype_bytes"], "kv_cache_layout": _kv_cache_layout(vllm_config),
                 "head_size": flat["head_size"], "num_heads": heads}
    if log_config and parallel["rank"] == 0:
        print("\n" + format_config_table({"parallel": parallel, "attention": attention}) + "\n")
    return KvbmVllmConfig(parallel, attention)
