"""``kvbm.vllm.sched_output``: vLLM's SchedulerOutput reduced to the connector's step view."""

from kvbm_b200.connector.vllm_connector import process_scheduler_output  # noqa: F401
