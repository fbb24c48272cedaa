"""Cross-parallelism (heterogeneous tensor parallelism) KV planning.

KV is sharded by KV head across TP ranks; two instances with different TP
degrees exchange blocks by slicing the head axis. For local TP ``L``,
remote TP ``R`` and ``G`` global KV heads:

* ``L == R``: local rank i <-> remote rank i, no slicing;
* ``L < R`` (``N = R / L``): local rank i receives from remote ranks
  ``i*N .. i*N+N-1``; remote rank j's ``G/R`` heads land at head offset
  ``(j - i*N) * G/R`` of local rank i;
* ``L > R`` (``N = L / R``): local rank i receives from remote rank ``i // N``
  the head sub-slice ``[(i % N) * G/L, (i % N + 1) * G/L)``.

Degrees must divide one another, shard axes and global extents must agree,
and pipeline parallelism must be 1 (layer slicing is reserved for it). The
plans drive the fused P->D kernel's head offsets, so the reshard happens in
the same launch as the NVLink store (no staging, no descriptor lists).

Parity: crates/kvbm-engine/src/p2p/dispatch.rs:1-47,195-397 (plan_pull,
compute_shards, build_axis_intersections) and p2p/parallelism.rs:28-492
(ParallelismTemplate, descriptor_for, validate_remote_metadata).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from ..common.tensor import AxisSlice, KvDim, intersect_axis


class CompatError(ValueError):
    pass


@dataclass(frozen=True)
class ParallelismTemplate:
    tp_size: int
    global_heads: int
    num_layers: int
    head_dim: int = 128
    page_size: int = 16
    dtype_width: int = 2
    pp_size: int = 1
    shard_axis: str = "head_count"
    mode: str = "tensor_parallel"

    @property
    def heads_per_rank(self) -> int:
        return self.global_heads // self.tp_size

    def descriptor_for(self, rank: int) -> dict:
        if not 0 <= rank < self.tp_size:
            raise ValueError(f"rank {rank} out of range for tp {self.tp_size}")
        h = self.heads_per_rank
        return {"rank": rank, "tp_size": self.tp_size, "head_range": (rank * h, (rank + 1) * h),
                "shard_axis": self.shard_axis, "global_heads": self.global_heads, "pp_size": self.pp_size,
                "num_layers": self.num_layers}


def validate(local: ParallelismTemplate, remote: ParallelismTemplate) -> None:
    if local.pp_size != 1 or remote.pp_size != 1:
        raise CompatError("pipeline parallelism is not supported (pp_size must be 1)")
    if local.shard_axis != remote.shard_axis:
        raise CompatError(f"shard axes differ: {local.shard_axis} vs {remote.shard_axis}")
    for f in ("global_heads", "num_layers", "head_dim", "page_size"):
        if getattr(local, f) != getattr(remote, f):
            raise CompatError(f"{f} differs: {getattr(local, f)} vs {getattr(remote, f)}")
    for t in (local, remote):
        if t.global_heads % t.tp_size:
            raise CompatError(f"{t.global_heads} heads are not divisible by tp {t.tp_size}")
    L, R = local.tp_size, remote.tp_size
    if max(L, R) % min(L, R):
        raise CompatError(f"tp degrees {L} and {R} do not divide one another")


@dataclass(frozen=True)
class Shard:
    remote_rank: int
    remote_head_offset: int   # first head within the remote rank's shard
    local_head_offset: int    # first head within the local rank's shard
    num_heads: int


@dataclass
class WorkerPullPlan:
    local_rank: int
    shards: list[Shard] = field(default_factory=list)


def plan_pull(local: ParallelismTemplate, remote: ParallelismTemplate) -> list[WorkerPullPlan]:
    """Per local rank: which remote ranks (and head slices) fill its shard."""
    validate(local, remote)
    L, R, G = local.tp_size, remote.tp_size, local.global_heads
    plans = []
    for i in range(L):
        mine = AxisSlice.shard(KvDim.HEAD, i, L, G)
        p = WorkerPullPlan(i)
        # remote ranks whose head windows overlap ours (contiguous run of ranks)
        for j in range(mine.start * R // G, (mine.end * R + G - 1) // G):
            inter = intersect_axis(AxisSlice.shard(KvDim.HEAD, j, R, G), mine)
            if inter is not None:
                p.shards.append(Shard(j, inter.src_local.start, inter.dst_local.start, len(inter)))
        plans.append(p)
    return plans


@dataclass(frozen=True)
class PushTarget:
    dst_rank: int
    src_head_offset: int
    dst_head_offset: int
    num_heads: int


def plan_push(src: ParallelismTemplate, dst: ParallelismTemplate) -> list[list[PushTarget]]:
    """Per source (prefill) rank: the destination (decode) ranks and head
    slices it stores into - the transpose of :func:`plan_pull` seen from the
    destination side."""
    pulls = plan_pull(dst, src)
    out: list[list[PushTarget]] = [[] for _ in range(src.tp_size)]
    for p in pulls:
        for s in p.shards:
            out[s.remote_rank].append(PushTarget(p.local_rank, s.remote_head_offset, s.local_head_offset,
                                                 s.num_heads))
    return out
