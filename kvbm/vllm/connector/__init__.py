"""``kvbm.vllm.connector``: KvbmConnector and PdConnector. vLLM is imported only
when a connector class is accessed."""


def __getattr__(name):
    if name in ("KvbmConnector", "KvbmConnectorMetadata"):
        from kvbm_b200.connector import vllm_connector

        return getattr(vllm_connector, name)
    if name == "PdConnector":
        from kvbm_b200.connector.pd import PdConnector

        return PdConnector
    raise AttributeError(name)
