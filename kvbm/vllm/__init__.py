"""vLLM integration (``kv_connector_module_path=kvbm.vllm.connector``), the prefill server
(``python -m kvbm.vllm.prefill``) and the supported-version check."""

from kvbm_b200._core import KvbmVllmConfig  # noqa: F401

from .version_check import version_check  # noqa: F401

__all__ = ["KvbmVllmConfig", "version_check"]
