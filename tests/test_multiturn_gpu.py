"""Multi-turn prefix reuse through the connector with G1 capped: later turns
must hit the shared prefix (G1 or G2) and onboard spilled blocks from G2."""

import argparse

import pytest

pytestmark = pytest.mark.gpu

from kvbm_b200.bench.multiturn_bench import run


def test_multiturn_spill_reuses_prefix_from_g2():
    a = argparse.Namespace(sessions=6, turns=3, prefix=64, gen=4, layers=2, g1_fraction=0.2, tiny=True, batch=4)
    r = run(a)
    assert r["hit_g2"] > 0, r
    assert r["hit_g1"] + r["hit_g2"] > 0.3 * r["total_prompt"]
    assert r["onboard_bytes"] > 0 and r["onboard_ms"] > 0
    assert len(r["ttft"]) == 18
