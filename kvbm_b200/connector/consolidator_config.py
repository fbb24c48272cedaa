"""When a vLLM scheduler's connector runs the KV-event consolidator, and on which endpoints.

The consolidator (``kvbm_b200.consolidator.service``) merges vLLM's own G1
events with the block manager's G2/G3 presence events into one deduplicated
stream for a KV-aware router. A scheduler-role connector starts it when:

* ``DYN_KVBM_KV_EVENTS_ENABLE_CONSOLIDATOR`` is unset or truthy ("1", "true",
  "on", "yes");
* the engine's connector is ``KvbmConnector`` (directly, or as a child of
  ``PdConnector``);
* prefix caching is on (vLLM publishes block events only then);
* vLLM publishes KV events (``kv_events_config``), since that is the stream
  the consolidator subscribes to.

Endpoints: the consolidator subscribes to vLLM's KV-event endpoint (its
port offset by the data-parallel rank the way vLLM offsets it; ``*``
becomes ``127.0.0.1``) and publishes on the block manager's event port
(``DYN_KVBM_LEADER_ZMQ_PUB_PORT``, default 56001) plus 1000.
``DYN_KVBM_KV_EVENTS_CONSOLIDATOR_MODE`` selects ``dedup`` (default) or
``passthrough``.

Parity: python/kvbm/vllm/consolidator_config.py (the same environment
variables, port rule and enable conditions, so deployments configured for
the reference keep working).
"""

from __future__ import annotations

import logging
import os

log = logging.getLogger(__name__)

DEFAULT_LEADER_PUB_PORT = 56001
CONSOLIDATOR_PORT_OFFSET = 1000


def is_truthy(val: str) -> bool:
    return val.strip().lower() in ("1", "true", "on", "yes")


def get_consolidator_mode() -> str:
    mode = os.getenv("DYN_KVBM_KV_EVENTS_CONSOLIDATOR_MODE", "dedup").strip().lower()
    if mode in ("dedup", "passthrough"):
        return mode
    log.warning("DYN_KVBM_KV_EVENTS_CONSOLIDATOR_MODE=%r is not dedup or passthrough; using dedup", mode)
    return "dedup"


def _uses_kvbm(ktc) -> bool:
    name = getattr(ktc, "kv_connector", None)
    if name == "KvbmConnector":
        return True
    if name == "PdConnector":
        kids = (getattr(ktc, "kv_connector_extra_config", None) or {}).get("connectors", [])
        return any(k.get("kv_connector") == "KvbmConnector" for k in kids)
    return False


def should_enable_consolidator(vllm_config) -> bool:
    if not is_truthy(os.getenv("DYN_KVBM_KV_EVENTS_ENABLE_CONSOLIDATOR", "true")):
        log.info("KV-event consolidator disabled by DYN_KVBM_KV_EVENTS_ENABLE_CONSOLIDATOR")
        return False
    ktc = getattr(vllm_config, "kv_transfer_config", None)
    if ktc is None or not _uses_kvbm(ktc):
        return False
    if not getattr(getattr(vllm_config, "cache_config", None), "enable_prefix_caching", False):
        log.warning("KV-event consolidator needs prefix caching (vLLM publishes no block events without it)")
        return False
    if getattr(vllm_config, "kv_events_config", None) is None:
        log.warning("KV-event consolidator needs vLLM's kv_events_config (--kv-events-config) to subscribe to")
        return False
    return True


def _offset_port(endpoint: str, dp_rank: int) -> str:
    """vLLM's per-data-parallel-rank endpoint: tcp ports shift by the rank, inproc names get a suffix."""
    if not endpoint or dp_rank == 0:
        return endpoint
    if "inproc" in endpoint:
        return f"{endpoint}_dp{dp_rank}"
    base, _, port = endpoint.rpartition(":")
    return f"{base}:{int(port) + dp_rank}"


def get_consolidator_endpoints(vllm_config) -> tuple[str, str, str] | None:
    """(vLLM event endpoint, output bind endpoint, output connect endpoint), or None when disabled."""
    if not should_enable_consolidator(vllm_config):
        return None
    dp = int(getattr(vllm_config.parallel_config, "data_parallel_rank", 0) or 0)
    if dp != 0:
        log.warning("the consolidator follows data-parallel rank 0's events only (this is rank %d)", dp)
        dp = 0
    vllm_ep = _offset_port(vllm_config.kv_events_config.endpoint, dp).replace("*", "127.0.0.1")
    port = int(os.getenv("DYN_KVBM_LEADER_ZMQ_PUB_PORT", str(DEFAULT_LEADER_PUB_PORT))) + CONSOLIDATOR_PORT_OFFSET
    if port > 65535:
        raise ValueError(f"consolidator port {port} exceeds 65535: lower DYN_KVBM_LEADER_ZMQ_PUB_PORT")
    return vllm_ep, f"tcp://0.0.0.0:{port}", f"tcp://127.0.0.1:{port}"
