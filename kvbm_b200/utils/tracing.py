"""Tracing: NVTX ranges on pipeline stages and a structured audit log.

* ``nvtx_range(name)`` marks a region for Nsight Systems / ncu (no-op when
  CUDA or NVTX is unavailable, or when ``KVBM_NVTX=0``).
* ``audit(event, **fields)`` writes one JSON line to the ``kvbm_audit``
  logger (session and worker lifecycle events), which external tools parse
  to reconstruct transfers.
* ``init_logging()`` configures log levels from ``KVBM_LOG`` / ``DYN_LOG``
  (default ``error``) unless ``KVBM_SKIP_LOG_INIT`` is set.

Parity: crates/kvbm-engine/src/audit.rs (kvbm_audit target),
tiering/offload/mod.rs:85-95 (nvtx feature), src/lib.rs:11-51 (log init
from RUST_LOG / DYN_LOG, KVBM_SKIP_LOG_INIT).
"""

from __future__ import annotations

import contextlib
import json
import logging
import os
import time

audit_log = logging.getLogger("kvbm_audit")
_NVTX = os.environ.get("KVBM_NVTX", "1") != "0"


@contextlib.contextmanager
def nvtx_range(name: str):
    pushed = False
    if _NVTX:
        try:
            import torch

            if torch.cuda.is_available():
                torch.cuda.nvtx.range_push(name)
                pushed = True
        except Exception:  # noqa: BLE001 - tracing must never break the caller
            pushed = False
    try:
        yield
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()


def audit(event: str, **fields) -> None:
    if audit_log.isEnabledFor(logging.INFO):
        audit_log.info(json.dumps({"ts": time.time(), "event": event, **fields}, default=str))


def init_logging() -> None:
    if os.environ.get("KVBM_SKIP_LOG_INIT"):
        return
    level = (os.environ.get("KVBM_LOG") or os.environ.get("DYN_LOG") or "error").upper()
    logging.basicConfig(level=getattr(logging, level, logging.ERROR),
                        format="%(asctime)s %(levelname)s %(name)s %(message)s")
