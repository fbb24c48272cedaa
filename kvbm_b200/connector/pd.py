"""PdConnector: the block manager first, a P/D transfer connector second.

vLLM's MultiConnector runs several connectors side by side; this one pairs
the KV block manager (prefix reuse, G2/G3 tiers; LMCache is accepted in its
place) with a prefill/decode transfer connector (vLLM's NIXL connector), so
a disaggregated deployment through NIXL keeps the block manager's cache
tiers. On one NVLink box the block manager's own conditional-disaggregation
path (``kvbm_b200.serving.pd``: dispatch through the connector leader,
pushes from the connector worker) does the P->D transfer without a second
connector.

Behaviour kept from the reference:

* exactly two children; the first must be ``KvbmConnector`` (or vLLM's
  LMCache connector when it is installed), the second ``NixlConnector``;
* handshake metadata is composite: each child's handshake travels in its
  own field (:class:`PdHandshakeMetadata`) and is routed back to that child
  only; a bare (non-composite) handshake is NIXL's (older senders);
* the first child alone answers ``get_num_new_matched_tokens``; on
  ``update_state_after_alloc`` the second child sees no blocks and no
  external tokens, so only the block manager loads prefixes;
* per-step metadata is one entry per child, bound to that child.

Parity: python/kvbm/vllm/connector/pd.py:57-140 (PdConnector,
PdHandshakeMetadata, PdConnectorMetadata).
"""

from __future__ import annotations


def __getattr__(name):
    if name in ("PdConnector", "PdHandshakeMetadata", "PdConnectorMetadata", "validate_children"):
        return _define()[name]
    raise AttributeError(name)


def _nixl_class():
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.nixl import NixlConnector
    except ImportError:  # before vLLM 0.19.1 the NIXL connector was one module
        from vllm.distributed.kv_transfer.kv_connector.v1.nixl_connector import NixlConnector
    return NixlConnector


def _define() -> dict:
    g = globals()
    if "_PD" in g:
        return g["_PD"]
    from dataclasses import dataclass

    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorHandshakeMetadata
    from vllm.distributed.kv_transfer.kv_connector.v1.multi_connector import (MultiConnector,
                                                                              MultiKVConnectorMetadata)

    from . import vllm_connector

    first_types = [vllm_connector.__getattr__("KvbmConnector")]
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.lmcache_connector import LMCacheConnectorV1

        first_types.append(LMCacheConnectorV1)
    except ImportError:
        pass

    @dataclass
    class PdConnectorMetadata(MultiKVConnectorMetadata):
        pass

    @dataclass
    class PdHandshakeMetadata(KVConnectorHandshakeMetadata):
        """Each child's handshake in its own field, routed back to that child only."""

        kvbm_metadata: KVConnectorHandshakeMetadata | None
        nixl_metadata: KVConnectorHandshakeMetadata | None

    class PdConnector(MultiConnector):
        """MultiConnector of the KV block manager (first) and NIXL (second)."""

        second_type = None  # resolved on first construction (NIXL import is slow)

        def __init__(self, vllm_config, role, kv_cache_config=None):
            super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)
            validate_children(self._connectors)

        def set_xfer_handshake_metadata(self, metadata) -> None:
            kvbm_meta, nixl_meta = route_handshake(metadata, PdHandshakeMetadata)
            if kvbm_meta and hasattr(self._connectors[0], "set_xfer_handshake_metadata"):
                self._connectors[0].set_xfer_handshake_metadata(kvbm_meta)
            if nixl_meta:
                self._connectors[1].set_xfer_handshake_metadata(nixl_meta)

        def get_handshake_metadata(self):
            a = self._connectors[0].get_handshake_metadata()
            b = self._connectors[1].get_handshake_metadata()
            if a is None and b is None:
                return None
            return PdHandshakeMetadata(kvbm_metadata=a, nixl_metadata=b)

        def bind_connector_metadata(self, connector_metadata) -> None:
            if not isinstance(connector_metadata, MultiKVConnectorMetadata):
                raise TypeError(f"PdConnector metadata expected, got {type(connector_metadata).__name__}")
            super().bind_connector_metadata(connector_metadata)

        def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
            return self._connectors[0].get_num_new_matched_tokens(request, num_computed_tokens)

        def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
            self._connectors[0].update_state_after_alloc(request, blocks, num_external_tokens)
            self._connectors[1].update_state_after_alloc(request, blocks.new_empty(), 0)

        def build_connector_meta(self, scheduler_output):
            meta = PdConnectorMetadata(metadata=tuple(c.build_connector_meta(scheduler_output)
                                                      for c in self._connectors))
            if self._extra_async_saves:
                meta.extra_async_saves = self._extra_async_saves
                self._extra_async_saves = {}
            return meta

    def validate_children(children) -> None:
        if len(children) != 2:
            raise ValueError(f"PdConnector requires exactly two connectors (got {len(children)})")
        if not isinstance(children[0], tuple(first_types)):
            names = " or ".join(t.__name__ for t in first_types)
            raise TypeError(f"Expected first connector to be {names}, got {type(children[0]).__name__}")
        if PdConnector.second_type is None:
            PdConnector.second_type = _nixl_class()
        if not isinstance(children[1], PdConnector.second_type):
            raise TypeError(f"Expected second connector to be NixlConnector, got {type(children[1]).__name__}")

    g["_PD"] = {"PdConnector": PdConnector, "PdHandshakeMetadata": PdHandshakeMetadata,
                "PdConnectorMetadata": PdConnectorMetadata, "validate_children": validate_children}
    return g["_PD"]


def route_handshake(metadata: dict, composite_type) -> tuple[dict, dict]:
    """Split per-rank handshakes into (block manager's, NIXL's); a non-composite entry is NIXL's."""
    kvbm_meta, nixl_meta = {}, {}
    for rank, m in metadata.items():
        if isinstance(m, composite_type):
            if m.kvbm_metadata is not None:
                kvbm_meta[rank] = m.kvbm_metadata
            if m.nixl_metadata is not None:
                nixl_meta[rank] = m.nixl_metadata
        else:
            nixl_meta[rank] = m
    return kvbm_meta, nixl_meta
