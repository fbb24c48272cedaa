"""Replicated-data broadcast across two GPUs: the NCCL baseline and the P2P
fan-out (rank 0 stores into the peer's pool over NVLink, flag-signalled).
Runs as two spawned processes, one per GPU, with a short process-group
timeout; every device wait is bounded."""

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

    from kvbm_b200.parallel.collectives import NcclCollectives, P2PFanoutCollectives
    from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
    from kvbm_b200.physical.verify import FillPattern, checksum_blocks, fill_blocks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cfg = LayoutConfig.for_model(16, 3, 4, 128, 16)
    g1 = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, zero=True)
    if rank == 0:
        fill_blocks(g1, [1, 2, 3], FillPattern.RANDOM, seed=7)
    want = [None]
    if rank == 0:
        want[0] = checksum_blocks(g1, [1, 2, 3])
    dist.broadcast_object_list(want, src=0)
    res = {}
    for name, cls in (("nccl", NcclCollectives), ("p2p", P2PFanoutCollectives)):
        if rank != 0:
            g1._flat().zero_()
        torch.cuda.synchronize()
        dist.barrier()
        coll = cls(g1)
        coll.broadcast([1, 2, 3], [5, 6, 7])
        torch.cuda.synchronize()
        if name == "p2p":
            coll.check()
        res[name] = checksum_blocks(g1, [5, 6, 7]) == want[0] if rank else True
        dist.barrier()
    out.put((rank, res))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_replicated_broadcast_nccl_and_p2p():
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
            r, res = out.get(timeout=180)
            results[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results[1] == {"nccl": True, "p2p": True}
