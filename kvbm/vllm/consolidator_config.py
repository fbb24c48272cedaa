"""``kvbm.vllm.consolidator_config``: when the scheduler runs the KV-event consolidator, and where."""

from kvbm_b200.connector.consolidator_config import (get_consolidator_endpoints, get_consolidator_mode,  # noqa: F401
                                                     is_truthy, should_enable_consolidator)
