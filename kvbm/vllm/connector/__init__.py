"""``kvbm.vllm.connector``: KvbmConnector and PdConnector. vLLM is imported only
when a connector class is accessed."""


def __getattr__(name):
    if name in ("KvbmConnector", "KvbmConnectorMetadata", "KvbmConnectorWorkerMetadata"):
        from kvbm_b200.connector import vllm_connector

        return getattr(vllm_connector, name)
    if name in ("PdConnector", "PdConnectorMetadata", "PdHandshakeMetadata"):
        from kvbm_b200.connector import pd

        return getattr(pd, name)
    raise AttributeError(name)
