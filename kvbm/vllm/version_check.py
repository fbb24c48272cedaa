"""``kvbm.vllm.version_check``: refuse vLLM versions outside the tested range
(``KVBM_SKIP_VLLM_VERSION_CHECK=1`` bypasses)."""

from kvbm_b200.connector.config import check_vllm_version as version_check  # noqa: F401
