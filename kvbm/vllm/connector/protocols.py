"""``kvbm.vllm.connector.protocols``: the vLLM scheduler-output fields the connector reads."""

from kvbm_b200.connector.vllm_connector import (CachedRequestDataProtocol, NewRequestDataProtocol,  # noqa: F401
                                                SchedulerOutputProtocol)
