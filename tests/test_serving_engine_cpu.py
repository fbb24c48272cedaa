"""The serving engine's scheduling on CPU: a stand-in model and connector
worker (no GPU), the real connector leader, conditional disaggregation
between a decode engine and a prefill engine over an in-process plane.
Checks the request lifecycle the driver harness relies on: remote prefill ->
received -> decode -> finished, delayed frees until the push is reported,
pipelined waves, local prefill, and a tensor-parallel plan broadcast."""

import pytest
import torch

from kvbm_b200.connector.leader import REMOTE_DECODE_KEY, ConnectorLeader
from kvbm_b200.connector.protocol import ConnectorMetadata
from kvbm_b200.engine.cd import ConditionalDisagg, InflightBudget, SelectionPolicy
from kvbm_b200.engine.cd_plane import LocalPrefillPlane
from kvbm_b200.engine.leader import InstanceLeader
from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.serving import engine as E


class FakeEvent:
    def __init__(self, *a, **k):
        pass

    def record(self, *a):
        pass

    def query(self):
        return True

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 1.0


class FakeStream:
    def __init__(self, *a, **k):
        pass


class FakeCfg:
    kv_heads, heads, head_dim, layers = 2, 4, 16, 2


class FakeModel:
    """Prefill and decode that only call the layer hooks and return fixed tokens."""

    def __init__(self):
        self.device = torch.device("cpu")
        self.cfg = FakeCfg()
        self.prefills, self.decodes = [], 0

    def allocate_pool(self, n, page):
        return object()

    def prefill(self, tokens, pool, ids, start_pos=0, on_layer_done=None, on_layer_start=None):
        self.prefills.append((int(tokens.numel()), start_pos))
        for l in range(self.cfg.layers):
            if on_layer_start:
                on_layer_start(l)
            if on_layer_done:
                on_layer_done(l)
        return torch.tensor([7])

    def decode_step(self, tok, pos, pool, table, seq_lens, splits):
        self.decodes += 1
        return (pos.long() % 100) + 1000


class FakeWorker:
    """Connector worker stand-in: pushes land in the decode worker's mailbox dict immediately."""

    mailboxes: dict = {}

    def __init__(self, instance):
        self.instance = instance
        self.meta = None
        self.pending_recv = {}
        self.pushed = []
        self.sending_pending = set()

    def bind_connector_metadata(self, raw):
        self.meta = ConnectorMetadata.decode(raw)

    def clear_connector_metadata(self):
        self.meta = None

    def start_load_kv(self):
        for op in self.meta.recv:
            self.pending_recv[op.req_id] = op

    def wait_for_layer_load(self, l):
        pass

    def save_kv_layer(self, l, requests=None):
        pass

    def wait_for_save(self):
        for op in self.meta.push:
            self.pushed.append(op)
            if op.final:
                FakeWorker.mailboxes[(op.peer, op.slot)] = op.seq

    def get_finished(self, finished):
        recving = {r for r, op in self.pending_recv.items()
                   if FakeWorker.mailboxes.get((self.instance, op.slot)) == op.seq}
        for r in recving:
            del self.pending_recv[r]
        self.sending_pending |= set(finished)
        sending, self.sending_pending = self.sending_pending, set()
        return sending, recving

    def build_connector_worker_meta(self):
        return None

    def get_block_ids_with_load_errors(self):
        return set()


@pytest.fixture(autouse=True)
def _no_cuda(monkeypatch):
    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.cuda, "Stream", FakeStream)
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    monkeypatch.setattr(E.llama_ops, "decode_splits", lambda *a, **k: 1)
    FakeWorker.mailboxes = {}


def make_pair(concurrency=3, gen=4):
    plane = LocalPrefillPlane()
    dl = ConnectorLeader(InstanceLeader.scheduler_side(BlockManager(1, 16, "lru", Tier.G2)), 16,
                         offload_enabled=False, cd=ConditionalDisagg(SelectionPolicy("always"), InflightBudget(8)),
                         plane=plane, prefill_target=2, instance_id=1, mailbox_slots=8)
    pl = ConnectorLeader(InstanceLeader.scheduler_side(BlockManager(1, 16, "lru", Tier.G2)), 16,
                         offload_enabled=False, instance_id=2)
    dec = E.LLMEngine(FakeModel(), E.EngineConfig(num_gpu_blocks=64, max_num_seqs=concurrency, max_model_len=256,
                                                  max_tokens=gen, use_graphs=False), dl, FakeWorker(1))
    pre = E.LLMEngine(FakeModel(), E.EngineConfig(num_gpu_blocks=32, max_num_seqs=1, max_model_len=256,
                                                  max_tokens=gen, use_graphs=False), pl, FakeWorker(2))
    return plane, dec, pre


def pump(plane, dec, pre, limit=500):
    for _ in range(limit):
        for d in plane.poll(2):
            params = dict(d["params"])
            params[REMOTE_DECODE_KEY] = d["decode"]
            pre.add_request(E.Request(d["request_id"], torch.from_numpy(d["tokens"].copy()), max_tokens=1,
                                      kv_transfer_params=params))
        while pre.has_unfinished() or pre._delayed:
            pre.step()
        dec.step()
        if not dec.has_unfinished():
            return
    raise AssertionError("engines did not drain")


def test_remote_prefill_then_decode_lifecycle():
    plane, dec, pre = make_pair()
    reqs = [E.Request(f"r{i}", torch.arange(40 + 10 * i, dtype=torch.int32), max_tokens=4) for i in range(3)]
    for r in reqs:
        dec.add_request(r)
    pump(plane, dec, pre)
    for r in reqs:
        assert r.status == E.RequestStatus.FINISHED and r.output is not None and r.output.numel() == 4
        assert r.num_external_tokens == r.num_prompt_tokens
    # decode recomputed each last prompt token: positions S-1 .. S+2 -> tokens (pos % 100) + 1000
    assert reqs[0].output.tolist() == [1039, 1040, 1041, 1042]
    assert dec.leader.cd_stats["received"] == 3 and pre.leader.cd_stats["pushed_blocks"] == 3 + 4 + 4
    assert not pre._delayed and len(pre.free_blocks) == 31 and len(dec.free_blocks) == 63
    assert dec.model.prefills == []  # the decode engine never prefilled


def test_waves_pipelined_and_slots_reused():
    plane, dec, pre = make_pair(concurrency=2, gen=3)
    outs = []
    for w in range(3):
        reqs = [E.Request(f"w{w}i{i}", torch.arange(20, dtype=torch.int32), max_tokens=3) for i in range(2)]
        for r in reqs:
            dec.add_request(r)
        outs.append(reqs)
    pump(plane, dec, pre)
    assert all(r.output.tolist() == [1019, 1020, 1021] for w in outs for r in w)
    assert sorted(dec.free_slots) == [0, 1]


def test_local_prefill_when_policy_says_so():
    plane, dec, pre = make_pair()
    dec.leader.cd = ConditionalDisagg(SelectionPolicy("never"))
    r = E.Request("loc", torch.arange(33, dtype=torch.int32), max_tokens=3)
    dec.add_request(r)
    pump(plane, dec, pre)
    assert dec.model.prefills == [(33, 0)]
    assert r.output.tolist() == [7, 1033, 1034]  # the prefill's token, then decode steps at positions 33, 34


def _tp_rank(rank, port, q):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    import test_serving_engine_cpu as T
    from kvbm_b200.serving import engine as E
    from kvbm_b200.serving.tp import TpComm

    torch.cuda.Event, torch.cuda.Stream = T.FakeEvent, T.FakeStream
    torch.Tensor.pin_memory = lambda self: self
    E.llama_ops.decode_splits = lambda *a, **k: 1
    os.environ.setdefault("KVBM_LOCK_CHECK", "1")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=timedelta(seconds=60))
    try:
        tp = TpComm.create([0, 1], nccl=False)
        leader = None
        if rank == 0:
            leader = ConnectorLeader(InstanceLeader.scheduler_side(BlockManager(1, 16, "lru", Tier.G2)), 16,
                                     offload_enabled=False, num_workers=2)
        model = T.FakeModel()
        eng = E.LLMEngine(model, E.EngineConfig(num_gpu_blocks=32, max_num_seqs=2, max_model_len=128, max_tokens=3,
                                                use_graphs=False), leader, T.FakeWorker(9), tp=tp)
        if rank == 0:
            for i in range(3):
                eng.add_request(E.Request(f"t{i}", torch.arange(20 + i, dtype=torch.int32), max_tokens=3))
        outs = []
        while tp.broadcast(eng.has_unfinished() if rank == 0 else None):
            outs += [r.output.tolist() for r in eng.step()]
        q.put((rank, model.prefills, model.decodes, outs))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_ranks_run_the_scheduling_rank_plans():
    """Rank 0 schedules and broadcasts plans; rank 1 (no leader, no requests of its own) runs the
    same prefill chunks and decode steps on its shard; outputs come back on rank 0."""
    import socket
    import sys

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    sys.path.insert(0, __import__("os").path.dirname(__file__))
    procs = [ctx.Process(target=_tp_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r[0], r[1:]) for r in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=30)
    assert res[0][0] == res[1][0] == [(20, 0), (21, 0), (22, 0)]
    assert res[0][1] == res[1][1] > 0
    assert sorted(res[0][2]) == [[7, 1020, 1021], [7, 1021, 1022], [7, 1022, 1023]]
    assert res[1][2] == []


class TimeoutWorker(FakeWorker):
    """A decode worker whose mailbox word never lands: after ``polls`` get_finished calls it reports
    the receive done with the request's blocks as load errors (what the real worker does when the
    receive timeout expires)."""

    def __init__(self, instance, polls=3):
        super().__init__(instance)
        self.polls, self.seen, self.errors = polls, {}, set()

    def get_finished(self, finished):
        recving = set()
        for r, op in list(self.pending_recv.items()):
            self.seen[r] = self.seen.get(r, 0) + 1
            if self.seen[r] >= self.polls:
                recving.add(r)
                self.errors.update(op.g1_ids)
                del self.pending_recv[r]
        return set(finished), recving

    def get_block_ids_with_load_errors(self):
        out, self.errors = self.errors, set()
        return out


def test_dropped_remote_prefill_times_out_and_is_recomputed_locally():
    """The prefill instance never serves the dispatch (the message is dropped): the decode worker's
    receive gives up, reports the blocks as load errors, the engine prefills the prompt itself and the
    leader frees the in-flight budget and the mailbox slot."""
    plane = LocalPrefillPlane()
    dl = ConnectorLeader(InstanceLeader.scheduler_side(BlockManager(1, 16, "lru", Tier.G2)), 16,
                         offload_enabled=False, cd=ConditionalDisagg(SelectionPolicy("always"), InflightBudget(2)),
                         plane=plane, prefill_target=2, instance_id=1, mailbox_slots=2)
    model = FakeModel()
    dec = E.LLMEngine(model, E.EngineConfig(num_gpu_blocks=64, max_num_seqs=2, max_model_len=256, max_tokens=3,
                                            use_graphs=False), dl, TimeoutWorker(1))
    r = E.Request("lost", torch.arange(40, dtype=torch.int32), max_tokens=3)
    dec.add_request(r)
    for _ in range(50):
        dec.step()
        if not dec.has_unfinished():
            break
    assert len(plane.poll(2)) == 1  # it was dispatched, and nobody served it
    assert r.status == E.RequestStatus.FINISHED and r.load_failed
    assert model.prefills == [(40, 0)] and dec.stats["recomputed"] == 1
    assert r.output.tolist() == [7, 1040, 1041]
    assert dl.cd.budget.inflight == 0 and len(dl._mailbox_free) == 2 and dl.cd_stats["failed"] == 1
