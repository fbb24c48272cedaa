"""One-to-many fan-out through NVSwitch multicast (``multimem.st``) across
two GPUs: rank 0's blocks land in every rank's pool at the destination ids,
the group counter orders each rank's stream behind the copy, and a second
call over a layer range stays in sequence. Two spawned processes, one per
GPU; every device wait is bounded and both ranks always leave through the
same barrier, so no rank exits while the other still uses the multicast
object."""

import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank: int, world: int, port: int, out):
    import torch.distributed as dist

    from kvbm_b200.parallel.collectives import NvlsFanoutCollectives
    from kvbm_b200.physical.layout import LayoutConfig
    from kvbm_b200.physical.verify import FillPattern, checksum_blocks, fill_blocks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    res = {"supported": False}
    try:
        cfg = LayoutConfig.for_model(16, 3, 4, 128, 16)
        g1, handle, flag_off = NvlsFanoutCollectives.allocate_pool(cfg)
        mc = [None] * world
        dist.all_gather_object(mc, int(getattr(handle, "multicast_ptr", 0) or 0))
        if all(mc):
            res["supported"] = True
            coll = NvlsFanoutCollectives(g1, handle, flag_off, wait_ns=10_000_000_000)
            if rank == 0:
                fill_blocks(g1, [1, 2, 3, 9], FillPattern.RANDOM, seed=7)
            want = [checksum_blocks(g1, [1, 2, 3]) if rank == 0 else None]
            dist.broadcast_object_list(want, src=0)
            coll.broadcast([1, 2, 3], [5, 6, 7])
            torch.cuda.synchronize()
            coll.check()
            res["first"] = checksum_blocks(g1, [5, 6, 7]) == want[0]
            # second call: layers 1..2 of block 9 into block 12 (layer 0 of block 12 stays zero)
            coll.broadcast([9], [12], layer_range=(1, 3))
            torch.cuda.synchronize()
            coll.check()
            src = [g1.gather_blocks([9]).cpu() if rank == 0 else None]
            dist.broadcast_object_list(src, src=0)
            got = g1.gather_blocks([12]).cpu()
            res["layers"] = bool(torch.equal(got[:, 1:], src[0][:, 1:]) and not got[:, 0].any())
            res["seq"] = coll.seq
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        out.put((rank, res))
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multicast_fanout_two_gpus():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            r, res = out.get(timeout=240)
            results[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    if not results[0]["supported"]:
        pytest.skip("no NVLink multicast object on this platform")
    for r in (0, 1):
        assert results[r] == {"supported": True, "first": True, "layers": True, "seq": 2}, results


def _rank_replicated(rank: int, world: int, port: int, out):
    import torch.distributed as dist

    from kvbm_b200.engine.worker import Worker
    from kvbm_b200.logical.manager import Tier
    from kvbm_b200.parallel.collectives import NvlsFanoutCollectives, P2PFanoutCollectives, ReplicatedDataWorker
    from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
    from kvbm_b200.physical.verify import FillPattern, checksum_blocks, fill_blocks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    res = {}
    try:
        cfg = LayoutConfig.for_model(16, 3, 4, 128, 16)
        pools = {"p2p": KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, zero=True)}
        g1n, handle, off = NvlsFanoutCollectives.allocate_pool(cfg)
        mc = [None] * world
        dist.all_gather_object(mc, int(getattr(handle, "multicast_ptr", 0) or 0))
        if all(mc):
            pools["nvls"] = g1n
        for name, g1 in pools.items():
            worker = Worker(rank, g1, g2_blocks=8)
            coll = P2PFanoutCollectives(g1) if name == "p2p" else NvlsFanoutCollectives(g1, handle, off)
            rdw = ReplicatedDataWorker(worker, coll)
            if rank == 0:
                fill_blocks(worker.g2_layout, [2, 5], FillPattern.RANDOM, seed=11)
            want = [checksum_blocks(worker.g2_layout, [2, 5]) if rank == 0 else None]
            dist.broadcast_object_list(want, src=0)
            # rank 0 onboards G2 [2, 5] into its G1 [9, 3], then every rank receives G1 [9, 3]
            rdw.onboard([2, 5] if rank == 0 else None, [9, 3])
            torch.cuda.synchronize()
            coll.check()
            res[name] = checksum_blocks(g1, [9, 3]) == want[0]
            dist.barrier()
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        out.put((rank, res))
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_replicated_data_worker_onboards_on_rank0_and_fans_out():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_replicated, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            r, res = out.get(timeout=240)
            results[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results[0].get("p2p") and results[1].get("p2p"), results
    if "nvls" in results[0]:
        assert results[0]["nvls"] and results[1]["nvls"], results
