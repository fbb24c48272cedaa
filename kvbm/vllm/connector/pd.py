"""``kvbm.vllm.connector.pd``: PdConnector (block manager first, a transfer connector second)."""


def __getattr__(name):
    if name in ("PdConnector", "PdConnectorMetadata", "PdHandshakeMetadata"):
        from kvbm_b200.connector import pd

        return getattr(pd, name)
    raise AttributeError(name)
