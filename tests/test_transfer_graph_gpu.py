"""Copy-engine transfers replayed from captured CUDA graphs (cuda_graph_replay)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
from kvbm_b200.physical.transfer import TransferCapabilities, TransferManager


def test_ce_regions_replay_from_a_graph():
    cfg = LayoutConfig.for_model(16, 4, 8, 128, 16, torch.bfloat16)
    nhd = KvBlockLayout.OPERATIONAL_NHD
    g1 = KvLayout.allocate(cfg, "layer_separate", nhd)
    g2 = KvLayout.allocate(cfg, "fully_contiguous", nhd, location="pinned", zero=True)
    tm = TransferManager(device=0, capabilities=TransferCapabilities(cuda_graph_replay=True, prefer_copy_engine=True))
    h1, h2 = tm.register_layout(g1), tm.register_layout(g2)
    src, dst = [3, 4, 9], [0, 5, 6]
    for rep in range(3):
        for l in range(cfg.num_layers):
            g1.layer_view(l).normal_()  # new data each time: the replay must copy it again
        torch.cuda.synchronize()
        tm.execute_transfer(h1, src, h2, dst).wait()
        torch.cuda.synchronize()
        assert torch.equal(g2.gather_blocks(dst).cuda(), g1.gather_blocks(src))
    assert tm.stats["graph_captures"] == 1 and tm.stats["graph_replays"] == 3
    tm.close()
