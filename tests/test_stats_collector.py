"""Rolling pool statistics (CPU): rates, hit ratios and gradients between samples on a fake clock."""

from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.sequence import sequence_hashes
from kvbm_b200.utils.metrics import StatsCollector


def test_rates_ratios_gradients_and_window():
    t = [0.0]
    mgr = BlockManager(16, 4, "lru", Tier.G2)
    sc = StatsCollector(mgr, window_size=3, clock=lambda: t[0])
    assert sc.sample() is None  # disabled by default
    sc.set_enabled(True)
    first = sc.sample()
    assert first.allocation_rate == 0 and first.reset_pool_size == 16
    hs = sequence_hashes(list(range(16)), 4)
    held = mgr.register_mutable(mgr.allocate_blocks(4), hs)
    t[0] = 2.0
    s1 = sc.sample()
    assert s1.allocation_rate == 2.0 and s1.allocation_gradient == 1.0
    assert s1.inflight_immutable == 4 and s1.reset_pool_size == 12
    del held  # blocks go inactive
    got = mgr.match_blocks(hs[:2] + [12345])
    t[0] = 3.0
    s2 = sc.sample()
    assert s2.allocation_rate == 0.0 and s2.allocation_gradient == -2.0
    assert abs(s2.match_hit_rate - 2 / 3) < 1e-9
    assert s2.inflight_immutable == 2 and s2.inactive_pool_size == 2
    del got
    t[0] = 4.0
    sc.sample()
    assert len(sc.window(10)) == 3 and sc.window(1)[0] == sc.latest()
    assert sc.window(3)[0] == s1  # the first sample fell out of the window
