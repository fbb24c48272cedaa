"""Prefill/decode deployment on one node, built from serving engines and the
block manager's connector.

A :class:`PdInstance` is one serving instance (``LLMEngine`` +
``ConnectorLeader`` + ``ConnectorWorker``) in a role:

decode
    Users submit requests here. The connector's conditional-disaggregation
    policy sends a request's prefill to a prefill instance: GNMT reports the
    prompt as an asynchronous external load, USAA dispatches it over the
    prefill plane with the destination G1 block ids and a mailbox slot, and
    the worker reports it received once the prefill GPU's completion word
    lands in the host mailbox. The engine then recomputes the last prompt
    token as the request's first decode step.
prefill
    Serves the plane (the role of the reference's ``PrefillRouterHandler``
    dispatch lambda): every dispatch becomes a one-token request whose
    ``kv_transfer_params`` name the decode instance; the connector worker
    pushes its blocks into the decode pool in layer batches during the
    prefill pass (one fused transfer kernel launch per batch, stores over
    NVLink) and publishes the completion word behind the last push.

Both roles can live in one process on one GPU (colocated: in-process plane
and directory, the push is a local HBM copy) or in separate processes on
separate GPUs (plane and directory over the process group's key-value
store, pools mapped with CUDA IPC, mailboxes in named shared memory).

Parity: docs/conditional-pd.md and crates/kvbm-engine/src/remote/cd/* of
the reference (decode-side plan, prefill accept, availability), with the
NIXL pull of the prefill's G2 blocks replaced by the push into the decode
G1 pool; python/kvbm/vllm/prefill.py + src/hub/prefill_router.rs for the
prefill server role.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ..connector.leader import REMOTE_DECODE_KEY, ConnectorLeader
from ..connector.worker import ConnectorWorker
from ..engine.cd import ConditionalDisagg, InflightBudget, SelectionPolicy
from ..engine.leader import InstanceLeader
from ..logical.manager import BlockManager, Tier
from ..models.llama import LlamaConfig, LlamaModel
from ..utils.config import KvbmConfig
from .engine import EngineConfig, LLMEngine, Request


@dataclass
class PdConfig:
    model: LlamaConfig = field(default_factory=LlamaConfig.llama3_8b)
    concurrency: int = 32            # requests per wave and decode batch slots
    prompt_len: int = 8192
    gen_len: int = 256
    page_size: int = 16
    layer_batch: int = 8             # layers per push launch
    push_engine: str = "tma"
    push_bulk_peer: bool = True      # same-layout peer pushes as TMA bulk stores over NVLink
    prefill_requests: int = 4        # prefill G1 capacity, in requests
    decode_waves: int = 2            # decode G1 capacity, in waves
    selection: str = "always"        # CD policy on the decode instance: always | threshold | never
    min_remote_prefill_tokens: int = 512
    use_graphs: bool = True
    seed: int = 0
    recv_timeout_s: float = 300.0
    wire_dtype: str = "bf16"         # bf16 | fp8 (block-scaled e4m3 over NVLink, dequantised on arrival)

    @property
    def request_blocks(self) -> int:
        return math.ceil((self.prompt_len + self.gen_len - 1) / self.page_size)

    @property
    def prompt_blocks(self) -> int:
        return math.ceil(self.prompt_len / self.page_size)

    def kv_bytes_per_request(self) -> int:
        c = self.model
        return self.prompt_blocks * c.layers * 2 * self.page_size * c.kv_heads * c.head_dim * 2


class PdInstance:
    """One serving instance of a P/D deployment."""

    def __init__(self, role: str, model: LlamaModel, cfg: PdConfig, instance_id: int, plane, directory,
                 shared: bool = False, prefill_target: int | None = None, timing: bool = True, tp=None):
        if role not in ("prefill", "decode"):
            raise ValueError(role)
        self.role, self.model, self.cfg, self.instance_id = role, model, cfg, int(instance_id)
        self.plane = plane
        self.tp = tp
        tp_rank, tp_size = (tp.rank, tp.size) if tp is not None else (0, 1)
        bs = cfg.page_size
        kcfg = KvbmConfig.load({"transfer": {"layer_batch": cfg.layer_batch, "push_engine": cfg.push_engine,
                                             "push_bulk_peer": cfg.push_bulk_peer}}, env={}, system_toml=None)
        cd = None
        slots = 0
        if role == "decode":
            slots = cfg.decode_waves * cfg.concurrency
            cd = ConditionalDisagg(SelectionPolicy(cfg.selection, cfg.min_remote_prefill_tokens),
                                   InflightBudget(slots))
            nblocks = cfg.decode_waves * cfg.concurrency * cfg.request_blocks + 1
            max_seqs = cfg.concurrency
        else:
            nblocks = cfg.prefill_requests * cfg.prompt_blocks + 1
            max_seqs = 1
        g2 = BlockManager(1, bs, "lru", Tier.G2)
        self.leader = None
        if tp_rank == 0:
            self.leader = ConnectorLeader(InstanceLeader.scheduler_side(g2), bs, offload_enabled=False, cd=cd,
                                          plane=plane if role == "decode" else None, prefill_target=prefill_target,
                                          instance_id=self.instance_id, mailbox_slots=slots,
                                          recv_timeout_s=cfg.recv_timeout_s, num_workers=tp_size, tp_size=tp_size,
                                          directory=directory)
        self.worker = ConnectorWorker(kcfg, rank=tp_rank, device=model.device.index, block_size=bs)
        ecfg = EngineConfig(num_gpu_blocks=nblocks, block_size=bs, max_num_seqs=max_seqs,
                            max_num_batched_tokens=max(cfg.prompt_len, 2048),
                            max_model_len=cfg.prompt_len + cfg.gen_len, max_tokens=cfg.gen_len,
                            use_graphs=cfg.use_graphs and role == "decode")
        self.engine = LLMEngine(model, ecfg, self.leader, self.worker, tp=tp)
        self.worker.register_layout(self.engine.pool)
        self.worker.enable_disagg(self.instance_id, directory, mailbox_slots=slots, shared=shared,
                                  timing=timing and role == "prefill", tp_rank=tp_rank, tp_size=tp_size,
                                  wire_dtype="fp8" if cfg.wire_dtype == "fp8" and role == "decode" else None)
        self.served = 0

    def warmup(self) -> None:
        self.engine.warmup()

    # ----------------------------------------------------------- prefill
    def pull(self, wait_s: float = 0.0) -> int:
        """Prefill role: turn dispatches waiting on the plane into requests (waits up to ``wait_s`` for one).
        With tensor parallelism only the instance's rank 0 takes dispatches (it schedules)."""
        if self.tp is not None and self.tp.rank != 0:
            return 0
        got = self.plane.wait(self.instance_id, wait_s) if wait_s > 0 else self.plane.poll(self.instance_id)
        for d in got:
            prompt = torch.from_numpy(d["tokens"].copy()).pin_memory()
            params = dict(d["params"])
            params[REMOTE_DECODE_KEY] = d["decode"]
            self.engine.add_request(Request(d["request_id"], prompt, max_tokens=1, kv_transfer_params=params,
                                            salt=d.get("salt")))
        return len(got)

    def step(self) -> list[Request]:
        out = self.engine.step()
        self.served += len(out)
        return out

    def shutdown(self) -> None:
        self.engine.release_graphs()
        self.worker.shutdown()
