"""Control plane of a tensor-parallel serving instance.

A TP instance is ``size`` processes (one per GPU). Rank 0 of the instance
schedules: it admits requests, calls the connector's scheduler hooks and
builds each step's :class:`~kvbm_b200.serving.engine.StepPlan`. The plan is
broadcast to every rank of the instance, each rank runs it on its model
shard (the all-reduces inside the forward pass line up because every rank
runs the same chunks in the same order) and on its connector worker, and
the workers' reports are gathered back to rank 0, which counts a request as
received or sent once every rank has reported it.

The broadcast and gather travel over a gloo group of the instance's ranks;
the model's all-reduces over an NCCL group of the same ranks.

Parity: the reference's TP instance is one vLLM engine whose executor
broadcasts the scheduler output to its workers (vLLM's multiproc executor)
and whose connector leader fans block operations out to every rank
(crates/kvbm-engine/src/worker/group/spmd.rs:31); the worker outputs are
aggregated per request (vLLM's KVOutputAggregator).
"""

from __future__ import annotations

import torch.distributed as dist


class TpComm:
    """The ranks of one tensor-parallel instance: ``ranks`` are global ranks, ``rank`` this
    process's index among them."""

    def __init__(self, ranks: list[int], gloo_group, nccl_group=None):
        self.ranks = list(ranks)
        self.size = len(self.ranks)
        self.rank = self.ranks.index(dist.get_rank())
        self.gloo, self.nccl = gloo_group, nccl_group

    @classmethod
    def create(cls, ranks: list[int], timeout=None, nccl: bool = True) -> "TpComm":
        """Collective over the whole world: every process must call it with the same ``ranks``
        sequence of every instance, in the same order (process groups are created collectively).
        ``nccl=False`` skips the NCCL group (control-plane tests without GPUs)."""
        kw = {"timeout": timeout} if timeout is not None else {}
        gloo = dist.new_group(ranks, backend="gloo", **kw)
        ng = dist.new_group(ranks, backend="nccl", **kw) if nccl else None
        return cls(ranks, gloo, ng)

    def broadcast_plan(self, plan):
        box = [plan]
        dist.broadcast_object_list(box, src=self.ranks[0], group=self.gloo)
        return box[0]

    def gather_reports(self, report: dict) -> list[dict] | None:
        out = [None] * self.size if self.rank == 0 else None
        dist.gather_object(report, out, dst=self.ranks[0], group=self.gloo)
        return out

    def broadcast(self, obj):
        box = [obj]
        dist.broadcast_object_list(box, src=self.ranks[0], group=self.gloo)
        return box[0]


def create_instances(groups: list[list[int]], timeout=None) -> dict[int, TpComm]:
    """Build every instance's TpComm collectively; returns {global rank: its instance's TpComm}
    for the ranks this process belongs to (one entry)."""
    me = dist.get_rank()
    mine = {}
    for ranks in groups:
        kw = {"timeout": timeout} if timeout is not None else {}
        gloo = dist.new_group(ranks, backend="gloo", **kw)
        nccl = dist.new_group(ranks, backend="nccl", **kw)
        if me in ranks:
            mine[me] = TpComm(ranks, gloo, nccl)
    return mine
