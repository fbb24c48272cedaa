"""``kvbm.vllm.connector.leader``: the scheduler-side connector (framework-neutral core)."""

from kvbm_b200.connector.leader import ConnectorLeader as KvbmConnectorLeader  # noqa: F401
from kvbm_b200.connector.leader import KvbmRequest, SchedulerOutputLite  # noqa: F401
