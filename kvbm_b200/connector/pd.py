"""PdConnector: the block manager first, a P/D transfer connector second.

vLLM's MultiConnector runs several connectors side by side; this one pairs
the KV block manager (prefix reuse, G2/G3 tiers) with a prefill/decode
transfer connector (NIXL in stock vLLM deployments), so a disaggregated
deployment keeps KVBM's cache tiers. On one NVLink box the block manager's
own fused P->D path (``kvbm_b200.engine.disagg``) replaces the second
connector.

Parity: python/kvbm/vllm/connector/pd.py:57 (PdConnector(MultiConnector)).
"""

from __future__ import annotations


def __getattr__(name):
    if name == "PdConnector":
        return _define()
    raise AttributeError(name)


def _define():
    g = globals()
    if "_PdConnector" in g:
        return g["_PdConnector"]
    from vllm.distributed.kv_transfer.kv_connector.v1.multi_connector import MultiConnector

    class PdConnector(MultiConnector):
        """MultiConnector whose first connector must be the KV block manager."""

        def __init__(self, vllm_config, role, kv_cache_config=None):
            super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)

    g["_PdConnector"] = PdConnector
    return PdConnector
