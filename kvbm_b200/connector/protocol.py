"""Wire format of the per-step connector metadata (leader -> workers).

One msgpack map per scheduler step::

    {"step": n,
     "onboard": [[req_id, g2_ids, g1_ids], ...],      # G2 -> G1 before the pass
     "offload": [[req_id, g1_ids, g2_ids], ...],      # G1 -> G2 after the pass
     "stage":   [[req_id, g3_ids, g2_ids], ...],      # G3 -> G2 before the onboards
     "spill":   [[g2_ids, g3_ids], ...],              # G2 -> G3 after the offloads
     "push":    [[req_id, peer, src, dst, slot, seq, final, peer_tp], ...],
     "recv":    [[req_id, slot, seq, g1_ids, timeout_s, contributors], ...],
     "pull":    [[pull_id, pools, src_ids, g2_ids], ...],
     "fetch":   [[req_id, hashes, g2_ids], ...],          # G4 -> G2 before the onboards
     "store":   [[g2_ids, hashes], ...],                  # G2 -> G4 (uploads, reported per step)
     "evict":   [req_id, ...]}

``push`` / ``recv`` carry conditional disaggregation: a prefill worker
pushes the listed G1 blocks of a request into the decode instance ``peer``
(its G1 pool mapped over NVLink) layer batch by layer batch while the
forward pass runs, and after the pass publishes ``seq`` in mailbox ``slot``
of that instance (``final``); the decode worker watches that mailbox slot
and reports the request as received once the value lands.

``pull`` carries remote search: each worker copies ``src_ids`` of another
instance's G2 pool (``pools[rank]``, a shared-memory pool on this node) into
``g2_ids`` of its own G2 pool and reports ``pull_id`` in its worker
metadata; the leader registers those G2 blocks once every worker has.

Parity: crates/kvbm-connector/src/connector/leader/mod.rs:551
(serialize_metadata, JSON WireMetadata{plan, control}); msgpack here.
crates/kvbm-protocols/src/disagg.rs:167 (RemotePrefillParams) for what a
remote prefill carries.
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
class StageOp:
    """G3 -> G2 for blocks a later onboard of the same step reads."""

    req_id: str
    g3_ids: list[int]
    g2_ids: list[int]


@dataclass
class SpillOp:
    """G2 -> G3 copy of blocks the leader registered in G3 (the G2 -> G3 chain)."""

    g2_ids: list[int]
    g3_ids: list[int]


@dataclass
class PushOp:
    """Prefill side: store ``src_ids`` (local G1) into ``dst_ids`` of instance ``peer``'s G1 pool."""

    req_id: str
    peer: int
    src_ids: list[int]
    dst_ids: list[int]
    slot: int
    seq: int
    final: bool
    peer_tp: int = 1          # TP degree of the decode instance (its ranks hold head shards)


@dataclass
class RecvOp:
    """Decode side: ``g1_ids`` of ``req_id`` arrive from a remote prefill; done when mailbox ``slot`` reads ``seq``."""

    req_id: str
    slot: int
    seq: int
    g1_ids: list[int]
    timeout_s: float = 60.0
    contributors: int = 1     # prefill ranks whose pushes fill one decode rank's shard


@dataclass
class FetchOp:
    """G4 -> G2: read the objects of ``hashes`` (this worker's rank keys) into ``g2_ids`` before the
    onboards of the same step."""

    req_id: str
    hashes: list[int]
    g2_ids: list[int]


@dataclass
class StoreOp:
    """G2 -> G4: upload registered G2 blocks ``g2_ids`` under ``hashes`` (this worker's rank keys)."""

    g2_ids: list[int]
    hashes: list[int]


@dataclass
class PullOp:
    """Remote search: copy another instance's G2 blocks ``src_ids`` into this instance's ``g2_ids``."""

    pull_id: int
    pools: list           # the holder's G2 pool exports, one per worker rank
    src_ids: list[int]
    g2_ids: list[int]


@dataclass
class ConnectorMetadata:
    step: int = 0
    onboard: list[OnboardOp] = field(default_factory=list)
    offload: list[OffloadOp] = field(default_factory=list)
    evict: list[str] = field(default_factory=list)
    stage: list[StageOp] = field(default_factory=list)
    spill: list[SpillOp] = field(default_factory=list)
    push: list[PushOp] = field(default_factory=list)
    recv: list[RecvOp] = field(default_factory=list)
    pull: list[PullOp] = field(default_factory=list)
    fetch: list[FetchOp] = field(default_factory=list)
    store: list[StoreOp] = field(default_factory=list)

    def encode(self) -> bytes:
        return msgpack.packb({
            "step": self.step,
            "onboard": [[o.req_id, o.g2_ids, o.g1_ids] for o in self.onboard],
            "offload": [[o.req_id, o.g1_ids, o.g2_ids] for o in self.offload],
            "evict": self.evict,
            "stage": [[o.req_id, o.g3_ids, o.g2_ids] for o in self.stage],
            "spill": [[o.g2_ids, o.g3_ids] for o in self.spill],
            "push": [[o.req_id, o.peer, o.src_ids, o.dst_ids, o.slot, o.seq, o.final, o.peer_tp]
                     for o in self.push],
            "recv": [[o.req_id, o.slot, o.seq, o.g1_ids, o.timeout_s, o.contributors] for o in self.recv],
            "pull": [[o.pull_id, o.pools, o.src_ids, o.g2_ids] for o in self.pull],
            # hashes are 192-bit: sent as decimal strings
            "fetch": [[o.req_id, [str(h) for h in o.hashes], o.g2_ids] for o in self.fetch],
            "store": [[o.g2_ids, [str(h) for h in o.hashes]] for o in self.store],
        }, use_bin_type=True)

    @classmethod
    def decode(cls, raw: bytes) -> "ConnectorMetadata":
        d = msgpack.unpackb(raw, raw=False)
        return cls(step=d["step"], onboard=[OnboardOp(*o) for o in d["onboard"]],
                   offload=[OffloadOp(*o) for o in d["offload"]], evict=list(d.get("evict", [])),
                   stage=[StageOp(*o) for o in d.get("stage", [])], spill=[SpillOp(*o) for o in d.get("spill", [])],
                   push=[PushOp(*o) for o in d.get("push", [])], recv=[RecvOp(*o) for o in d.get("recv", [])],
                   pull=[PullOp(*o) for o in d.get("pull", [])],
                   fetch=[FetchOp(r, [int(h) for h in hs], g) for r, hs, g in d.get("fetch", [])],
                   store=[StoreOp(g, [int(h) for h in hs]) for g, hs in d.get("store", [])])

    def empty(self) -> bool:
        return not (self.onboard or self.offload or self.evict or self.stage or self.spill or self.push or self.recv
                    or self.pull or self.fetch or self.store)
