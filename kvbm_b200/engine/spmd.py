"""Tensor-parallel worker group across processes (SPMD).

With tensor parallelism every rank holds its shard of every KV block (its
``num_kv_heads / tp`` heads) in its own G1, G2 and G3 pools, so every block
operation the leader decides - stage G3 -> G2, onboard G2 -> G1, offload
G1 -> G2, spill G2 -> G3 - runs once per rank, on the same block ids, each
rank moving its own heads.

* :class:`WorkerService` serves one rank's :class:`~kvbm_b200.engine.worker.Worker`
  over the messenger: transfers by tier, layer-wise onboards, the layout
  handshake.
* :class:`RemoteWorker` is the leader's proxy of one rank: each call is an
  RPC whose reply arrives once the rank's copy completed on its device, so
  its notification is a future.
* :class:`SpmdParallelWorkers` fans every op out to all ranks concurrently
  and aggregates the completions (the op is complete when every rank's part
  is); a rank that fails or does not answer fails the op.

Parity: crates/kvbm-engine/src/worker/group/spmd.rs:31 (SpmdParallelWorkers:
fan out every op to all ranks, aggregate notifications), worker/velo/
{service,client}.rs (VeloWorkerService / VeloWorkerClient), docs/worker-group.md.
"""

from __future__ import annotations

import concurrent.futures as cf

from ..logical.manager import Tier
from ..physical.transfer import TransferCompleteNotification
from .leader import ParallelWorkers

H_TRANSFER = "kvbm.worker.execute_local_transfer"
H_LAYERWISE = "kvbm.worker.start_layerwise_onboard"
H_LAYOUT = "kvbm.worker.layout"


class WorkerService:
    """One TP rank's worker behind the messenger."""

    def __init__(self, messenger, worker, rank: int):
        self.messenger, self.worker, self.rank = messenger, worker, rank
        messenger.register_handler(H_TRANSFER, self._transfer)
        messenger.register_handler(H_LAYERWISE, self._layerwise)
        messenger.register_handler(H_LAYOUT, self._layout)

    def _transfer(self, p: dict) -> dict:
        lr = tuple(p["layer_range"]) if p.get("layer_range") else None
        note = self.worker.execute_local_transfer(Tier(p["src"]), p["src_ids"], Tier(p["dst"]), p["dst_ids"],
                                                  layer_range=lr)
        note.wait(timeout=p.get("timeout"))
        return {"rank": self.rank, "ok": True, "blocks": len(p["src_ids"])}

    def _layerwise(self, p: dict) -> dict:
        self.worker.start_layerwise_onboard(p["g2_ids"], p["g1_ids"])
        return {"rank": self.rank, "ok": True}

    def _layout(self, _p) -> dict:
        g1 = self.worker.g1_layout.config
        return {"rank": self.rank, "num_heads": g1.num_heads, "num_layers": g1.num_layers,
                "bytes_per_block": g1.bytes_per_block}


class RemoteWorker:
    """Leader-side proxy of one TP rank's worker service."""

    def __init__(self, messenger, instance_id: int, rank: int, pool: cf.ThreadPoolExecutor | None = None,
                 timeout: float = 60.0):
        self.messenger, self.instance_id, self.rank = messenger, int(instance_id), rank
        self.timeout = timeout
        self._pool = pool or cf.ThreadPoolExecutor(max_workers=2, thread_name_prefix=f"kvbm-spmd-{rank}")

    def _rpc(self, handler: str, payload: dict) -> dict:
        r = self.messenger.call(self.instance_id, handler, payload, timeout=self.timeout)
        if not r or not r.get("ok"):
            raise RuntimeError(f"rank {self.rank}: {handler} failed: {r}")
        return r

    def execute_local_transfer(self, src_tier, src_ids, dst_tier, dst_ids, layer_range=None):
        payload = {"src": int(src_tier), "src_ids": list(map(int, src_ids)), "dst": int(dst_tier),
                   "dst_ids": list(map(int, dst_ids)), "layer_range": list(layer_range) if layer_range else None,
                   "timeout": self.timeout}
        return TransferCompleteNotification(future=self._pool.submit(self._rpc, H_TRANSFER, payload))

    def start_layerwise_onboard(self, g2_ids, g1_ids) -> None:
        self._rpc(H_LAYERWISE, {"g2_ids": list(map(int, g2_ids)), "g1_ids": list(map(int, g1_ids))})

    def layout(self) -> dict:
        return self.messenger.call(self.instance_id, H_LAYOUT, {}, timeout=self.timeout)


class SpmdParallelWorkers(ParallelWorkers):
    """The leader's handle on a TP group of worker processes."""

    def __init__(self, messenger, instances: list[int], timeout: float = 60.0):
        pool = cf.ThreadPoolExecutor(max_workers=max(2, 2 * len(instances)), thread_name_prefix="kvbm-spmd")
        super().__init__([RemoteWorker(messenger, iid, r, pool, timeout) for r, iid in enumerate(instances)])
        self._pool = pool

    def layouts(self) -> list[dict]:
        """Every rank's layout facts; ranks must agree on layers and block size (heads are the shard)."""
        ls = [w.layout() for w in self.workers]
        if len({(l["num_layers"], l["bytes_per_block"]) for l in ls}) > 1:
            raise ValueError(f"TP ranks disagree on their KV layout: {ls}")
        return ls

    def close(self) -> None:
        self._pool.shutdown(wait=False)
