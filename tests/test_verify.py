"""Checksums, fill patterns and the startup-benchmark cache (CPU parts)."""

import numpy as np
import torch

from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
from kvbm_b200.physical.verify import (FillPattern, StartupBenchmark, checksum_blocks, checksum_reference,
                                       fill_blocks)


def _host_pool(kind, bl, nb=6, dtype=torch.bfloat16):
    cfg = LayoutConfig.for_model(nb, 3, 4, 64, 16, dtype)
    probe = KvLayout._strides(cfg, kind, bl, True)
    t = torch.zeros(probe[-1], dtype=torch.uint8)
    return KvLayout.over_tensor(cfg, t, kind, bl), t


def test_checksum_is_layout_independent_and_content_sensitive():
    a, _ = _host_pool("fully_contiguous", KvBlockLayout.OPERATIONAL_NHD)
    b, _ = _host_pool("fully_contiguous", KvBlockLayout.OPERATIONAL_HND)
    fill_blocks(a, [0, 1, 2], FillPattern.RANDOM, seed=3)
    b.scatter_blocks([4, 5, 1], a.gather_blocks([0, 1, 2]))
    ca, cb = checksum_blocks(a, [0, 1, 2]), checksum_blocks(b, [4, 5, 1])
    assert ca == cb and len(set(ca)) == 3
    # one flipped bit changes the checksum; swapping two words changes it too
    g = a.gather_blocks([0])
    g.view(torch.int16).view(-1)[17] ^= 1
    assert checksum_reference(g[0]) != ca[0]
    g = a.gather_blocks([0])
    flat = g.view(torch.int32).view(-1)
    flat[[3, 4]] = flat[[4, 3]]
    if flat[3] != flat[4]:
        assert checksum_reference(g[0]) != ca[0]
    # a layer subrange is the checksum of that slice
    sub = checksum_blocks(a, [2], layer_begin=1, num_layers=2)[0]
    assert sub == checksum_reference(a.gather_blocks([2])[0, 1:3])


def test_fill_patterns_exact():
    a, _ = _host_pool("layer_separate", KvBlockLayout.OPERATIONAL_NHD)
    fill_blocks(a, [3, 5], FillPattern.BLOCK_ID)
    g = a.gather_blocks([3, 5]).float()
    assert (g[0] == 4).all() and (g[1] == 6).all()
    fill_blocks(a, [1], FillPattern.INDEX)
    v = a.gather_blocks([1])[0].float()  # [L, O, page, H, D]
    assert float(v[2, 1, 3, 2, 5]) == float((1 * 7 + 2 * 5 + 1 * 3 + 3 * 11 + 2 * 13 + 5) % 251)
    fill_blocks(a, [1], FillPattern.CONSTANT, value=2.5)
    assert (a.gather_blocks([1]).float() == 2.5).all()
    fill_blocks(a, [1], "zeros")
    assert not a.gather_blocks([1]).float().any()


def test_reference_matches_manual_definition():
    x = np.arange(8, dtype=np.uint32)
    m1, m2, gold = 0xBF58476D1CE4E5B9, 0x94D049BB133111EB, 0x9E3779B97F4A7C15
    mask = (1 << 64) - 1

    def mix(z):
        z = ((z ^ (z >> 30)) * m1) & mask
        z = ((z ^ (z >> 27)) * m2) & mask
        return z ^ (z >> 31)

    want = sum(mix(((i << 32) ^ int(w) ^ gold) & mask) for i, w in enumerate(x)) & mask
    assert checksum_reference(x) == want


def test_startup_benchmark_cache_roundtrip(tmp_path):
    a, _ = _host_pool("fully_contiguous", KvBlockLayout.OPERATIONAL_NHD)
    b, _ = _host_pool("fully_contiguous", KvBlockLayout.OPERATIONAL_HND)
    sb = StartupBenchmark(tmp_path / "bench.json")
    assert sb.lookup(a, b) is None
    assert sb.record(a, b, {"tile": 10.0, "tma": 30.0, "ce": 5.0}) == "tma"
    again = StartupBenchmark(tmp_path / "bench.json")
    assert again.lookup(a, b) == "tma" and again.lookup(b, a) is None
