"""NUMA-placed host pools on CPU: placement policy, first touch, layout allocation."""

import torch

from kvbm_b200.physical.layout import KvLayout, LayoutConfig
from kvbm_b200.physical.memory import NumaHostBuffer, bind_to_numa, gpu_numa_node, numa_node_of


def test_numa_buffer_on_node0_is_usable():
    b = NumaHostBuffer(3 * 4096 + 100, node=0, pin=False)
    t = b.tensor()
    assert t.numel() == b.nbytes and int(t.sum()) == 0  # first touch zero-fills
    t[:16] = 7
    assert int(b.tensor()[:16].sum()) == 7 * 16
    if b.numa_bound:  # the kernel accepted the policy: pages sit on node 0
        assert numa_node_of(b.ptr) == 0
    b.close()


def test_bind_rejects_bad_nodes():
    assert bind_to_numa(0, 4096, -1) is False
    assert bind_to_numa(0, 0, 0) is False


def test_gpu_numa_node_without_gpu():
    if not torch.cuda.is_available():
        assert gpu_numa_node() == -1


def test_layout_allocates_numa_pinned_pool():
    cfg = LayoutConfig(num_blocks=4, num_layers=2, outer_dim=2, page_size=16, inner_dim=16 * 2 * 64, dtype_width_bytes=2,
                       num_heads=2)
    lay = KvLayout.allocate(cfg, location="pinned", numa_node=0)
    assert lay.location == "pinned" and lay.nbytes >= cfg.bytes_per_block * 4
    lay.backing.tensor().view(torch.uint8)[:8] = 1
    assert int(lay.backing.tensor()[:8].sum()) == 8


def test_config_carries_g2_numa_placement():
    from kvbm_b200.utils.config import KvbmConfig

    cfg = KvbmConfig.load(env={"KVBM_CACHE_HOST_NUMA_NODE": "gpu", "KVBM_CACHE_HOST_HUGEPAGES": "true"})
    assert cfg.cache.host.numa_node == "gpu" and cfg.cache.host.hugepages is True
    cfg = KvbmConfig.load(env={"KVBM_CACHE_HOST_NUMA_NODE": "1"})
    assert cfg.cache.host.numa_node == 1 and cfg.cache.host.hugepages is False


def test_hugepage_buffer_falls_back_cleanly():
    b = NumaHostBuffer(5 << 20, node=0, hugepages=True, pin=False)
    assert b.hugepages in ("hugetlb", "thp", False)
    b.tensor()[:10] = 1
    assert int(b.tensor().sum()) == 10
    b.close()
