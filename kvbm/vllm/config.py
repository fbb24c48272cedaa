"""``kvbm.vllm.config``: the vLLM facts the connector sizes its pools from, and their table."""

from kvbm_b200.connector.config import extract_vllm_config_for_kvbm, format_config_table, kv_block_bytes  # noqa: F401
