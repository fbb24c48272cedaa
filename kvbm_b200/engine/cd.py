"""Conditional disaggregation (CD): decide per request whether to prefill
locally or on a remote prefill instance, within an in-flight budget.

* :class:`SelectionPolicy` - ``never``, ``always`` or ``threshold``: remote
  when the tokens that still need prefill (prompt - already computed -
  connector-provided) reach ``min_remote_prefill_tokens``;
* :class:`InflightBudget` - a compare-and-swap counter bounding concurrent
  remote prefills;
* the prefill router's breaker tier narrows decisions: warm halves the
  budget, hot forces local prefill;
* :class:`RemotePrefillParams` - what the decode side sends with the request
  (session id, initiator, decode endpoint, provided-token count, ...).

Parity: crates/kvbm-engine/src/remote/cd/{mod.rs:41-72 (DisaggConfig:
Never / unbounded budget / local fallback / drain poll 2 ms / watchdog 10 s),
policy.rs (SelectionPolicy, num_prefill_tokens = total - computed -
connector), budget.rs:16 (InflightBudget, TierCell)},
crates/kvbm-protocols/src/disagg.rs:167 (RemotePrefillParams).
"""

from __future__ import annotations

import enum
import threading
import uuid
from dataclasses import asdict, dataclass, field


class Decision(str, enum.Enum):
    LOCAL = "local"
    REMOTE = "remote"


@dataclass
class SelectionPolicy:
    kind: str = "never"                 # never | always | threshold
    min_remote_prefill_tokens: int = 512

    @staticmethod
    def num_prefill_tokens(total: int, computed: int, connector: int) -> int:
        return max(0, total - computed - connector)

    def decide(self, total: int, computed: int = 0, connector: int = 0) -> Decision:
        if self.kind == "never":
            return Decision.LOCAL
        if self.kind == "always":
            return Decision.REMOTE
        if self.kind == "threshold":
            n = self.num_prefill_tokens(total, computed, connector)
            return Decision.REMOTE if n >= self.min_remote_prefill_tokens else Decision.LOCAL
        raise ValueError(f"unknown selection policy {self.kind!r}")


class InflightBudget:
    def __init__(self, limit: int | None = None):
        self.limit = limit
        self._n = 0
        self._lock = threading.Lock()

    def try_reserve(self, limit_override: int | None = None) -> bool:
        lim = self.limit if limit_override is None else limit_override
        with self._lock:
            if lim is not None and self._n >= lim:
                return False
            self._n += 1
            return True

    def release(self) -> None:
        with self._lock:
            self._n = max(0, self._n - 1)

    @property
    def inflight(self) -> int:
        return self._n


@dataclass
class RemotePrefillParams:
    session_id: str = field(default_factory=lambda: uuid.uuid4().hex)
    initiator_instance_id: str = ""
    decode_endpoint: str = ""
    num_provided_tokens: int = 0
    window_start: int = 0
    provided_digest: str | None = None
    protocol_version: int = 1

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "RemotePrefillParams":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


class ConditionalDisagg:
    """Decode-side decision point (the GNMT hook asks it per new request)."""

    def __init__(self, policy: SelectionPolicy | None = None, budget: InflightBudget | None = None,
                 fallback: str = "local", metrics=None):
        self.policy = policy or SelectionPolicy()
        self.budget = budget or InflightBudget()
        self.fallback = fallback
        self.breaker_tier = 0  # 0 calm, 1 warm, 2 hot (pushed by the prefill router)
        self.metrics = metrics

    def decide(self, total: int, computed: int = 0, connector: int = 0) -> Decision:
        d = self.policy.decide(total, computed, connector)
        if d == Decision.REMOTE:
            if self.breaker_tier >= 2:
                d = Decision.LOCAL
            else:
                lim = self.budget.limit
                if self.breaker_tier == 1 and lim is not None:
                    lim = max(1, lim // 2)
                if not self.budget.try_reserve(lim):
                    d = Decision.LOCAL
        if self.metrics is not None:
            self.metrics.decisions[d.value] = self.metrics.decisions.get(d.value, 0) + 1
            if d == Decision.REMOTE:
                self.metrics.remote_tokens += SelectionPolicy.num_prefill_tokens(total, computed, connector)
        return d

    def finish_remote(self) -> None:
        self.budget.release()
