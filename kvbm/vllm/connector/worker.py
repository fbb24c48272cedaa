"""``kvbm.vllm.connector.worker``: the model-runner-side connector (framework-neutral core)."""

from kvbm_b200.connector.worker import ConnectorWorker as KvbmConnectorWorker  # noqa: F401
