"""Wire format of the per-step connector metadata (leader -> workers).

One msgpack map per scheduler step:
``{"step": n, "onboard": [[req_id, g2_ids, g1_ids], ...],
  "offload": [[req_id, g1_ids, g2_ids], ...], "evict": [...]}``.

Parity: crates/kvbm-connector/src/connector/leader/mod.rs:551
(serialize_metadata, JSON WireMetadata{plan, control}); msgpack here.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import msgpack


@dataclass
class OnboardOp:
    req_id: str
    g2_ids: list[int]
    g1_ids: list[int]


@dataclass
class OffloadOp:
    req_id: str
    g1_ids: list[int]
    g2_ids: list[int]


@dataclass
class ConnectorMetadata:
    step: int = 0
    onboard: list[OnboardOp] = field(default_factory=list)
    offload: list[OffloadOp] = field(default_factory=list)
    evict: list[str] = field(default_factory=list)

    def encode(self) -> bytes:
        return msgpack.packb({
            "step": self.step,
            "onboard": [[o.req_id, o.g2_ids, o.g1_ids] for o in self.onboard],
            "offload": [[o.req_id, o.g1_ids, o.g2_ids] for o in self.offload],
            "evict": self.evict,
        }, use_bin_type=True)

    @classmethod
    def decode(cls, raw: bytes) -> "ConnectorMetadata":
        d = msgpack.unpackb(raw, raw=False)
        return cls(step=d["step"], onboard=[OnboardOp(*o) for o in d["onboard"]],
                   offload=[OffloadOp(*o) for o in d["offload"]], evict=list(d.get("evict", [])))
