"""``kvbm.vllm.connector.base``: KvbmConnector and its metadata (vLLM imported on first access)."""


def __getattr__(name):
    if name in ("KvbmConnector", "KvbmConnectorMetadata", "KvbmConnectorWorkerMetadata"):
        from kvbm_b200.connector import vllm_connector

        return getattr(vllm_connector, name)
    raise AttributeError(name)
