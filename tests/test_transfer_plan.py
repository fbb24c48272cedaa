"""Transfer planner on CPU: classification, byte ranges against the layouts'
own addressing, coalescing, lowering rules, and the manager's plan cache."""

import ctypes as C
import itertools

import pytest
import torch

from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig
from kvbm_b200.physical.plan import (CopyOp, CopyPolicy, PlanKind, PreparedPlanCache, coalesce, lower, plan_copy,
                                     same_geometry)

NHD, HND, UNI = KvBlockLayout.OPERATIONAL_NHD, KvBlockLayout.OPERATIONAL_HND, KvBlockLayout.UNIVERSAL


def _cfg(nb=8, dtype=torch.bfloat16):
    return LayoutConfig.for_model(nb, 3, 2, 64, 16, dtype)


def _host(kind, bl, dtype=torch.bfloat16, nb=8):
    lay = KvLayout.allocate(_cfg(nb, dtype), kind, bl, location="pinned", numa_node=0)
    return lay


def test_coalesce_merges_only_doubly_contiguous_runs():
    ops = [CopyOp(0, 100, 10), CopyOp(10, 110, 10), CopyOp(20, 200, 10), CopyOp(30, 210, 5)]
    assert coalesce(ops) == [CopyOp(0, 100, 20), CopyOp(20, 200, 15)]


@pytest.mark.parametrize("src_kind,dst_kind", [("fully_contiguous", "fully_contiguous"),
                                               ("fully_contiguous", "layer_separate"),
                                               ("layer_separate", "fully_contiguous")])
def test_direct_ops_move_exactly_the_blocks(src_kind, dst_kind):
    a, b = _host(src_kind, NHD), _host(dst_kind, NHD)
    g = torch.Generator().manual_seed(1)
    for l in range(a.config.num_layers):
        v = a.layer_view(l)
        v.copy_(torch.randn(v.shape, generator=g).to(v.dtype))
    s_ids, d_ids = [1, 2, 3, 6], [4, 5, 6, 0]
    plan = plan_copy(a, s_ids, b, d_ids)
    assert plan.kind == PlanKind.DIRECT
    ops = plan.ops()
    assert sum(o.size for o in ops) == plan.bytes
    for o in ops:
        C.memmove(o.dst, o.src, o.size)
    assert torch.equal(b.gather_blocks(d_ids), a.gather_blocks(s_ids))
    if src_kind == dst_kind == "fully_contiguous":
        assert plan.whole_blocks and len(ops) == 2  # 1,2,3 -> 4,5,6 merge; 6 -> 0 alone


def test_layer_range_plans_chunks():
    a, b = _host("fully_contiguous", NHD), _host("fully_contiguous", NHD)
    plan = plan_copy(a, [0, 1], b, [2, 3], layer_range=(1, 3))
    assert plan.kind == PlanKind.DIRECT and not plan.whole_blocks and plan.unit == a.config.bytes_per_chunk
    assert plan.bytes == 2 * 2 * a.config.outer_dim * a.config.bytes_per_chunk


@pytest.mark.parametrize("why,kw", [
    ("dtype cast", dict(dst_dtype=torch.float8_e4m3fn)),
    ("block layout permute", dict(dst_bl=HND)),
    ("KV-head slice", dict(head_range=(0, 0, 1))),
])
def test_transforms_are_classified(why, kw):
    a = _host("fully_contiguous", NHD)
    b = _host("fully_contiguous", kw.get("dst_bl", NHD), kw.get("dst_dtype", torch.bfloat16))
    plan = plan_copy(a, [0], b, [1], head_range=kw.get("head_range"))
    assert plan.kind == PlanKind.TRANSFORM and plan.reason == why and plan.ops() == []


def _old_rules(src, dst, engine="auto", prefer_ce=False, layer_range=None, head_range=None, bench=None):
    """The engine choice as the transfer manager made it before the planner existed."""
    if engine != "auto":
        return engine
    if prefer_ce:
        return "ce"
    a, b = src.config, dst.config
    same = (src.kind == dst.kind == "fully_contiguous" and src.block_layout == dst.block_layout
            and src.dtype == dst.dtype and layer_range is None and head_range is None and same_geometry(src, dst)
            and src.block_stride == a.bytes_per_block and dst.block_stride == b.bytes_per_block)
    if same:
        return "pairs"
    if bench is not None:
        return bench
    return "tile" if src.dtype != dst.dtype else "tma"


def test_lowering_matches_the_previous_rules():
    pools = [_host(k, bl, dt) for k, bl, dt in itertools.product(
        ["fully_contiguous", "layer_separate"], [NHD, HND, UNI], [torch.bfloat16, torch.float8_e4m3fn])
        if not (k == "layer_separate" and bl == UNI)]
    for a, b in itertools.product(pools, pools):
        for hr, eng, ce, bench in [(None, "auto", False, None), ((0, 0, 1), "auto", False, None),
                                   (None, "tile", False, None), (None, "auto", True, None),
                                   (None, "auto", False, "tile")]:
            if hr is not None and a.block_layout == UNI:
                continue
            plan = plan_copy(a, [0, 1], b, [2, 3], head_range=hr)
            got = lower(plan, a, b, prefer_copy_engine=ce, engine=eng, bench_choice=bench).engine
            assert got == _old_rules(a, b, eng, ce, None, hr, bench), (a.kind, a.block_layout, b.block_layout)


def test_dma_check_uses_run_size():
    a, b = _host("fully_contiguous", NHD), _host("fully_contiguous", NHD)
    low = lower(plan_copy(a, [0], b, [1], layer_range=(0, 1)), a, b, policy=CopyPolicy(min_inner_bytes=1 << 30))
    assert low.dma_ok is False
    assert lower(plan_copy(a, [0], b, [1]), a, b).dma_ok is True  # whole blocks are >= 4 KiB


def test_manager_memoises_engine_choices():
    from kvbm_b200.physical.transfer import TransferManager, TransferOptions

    tm = TransferManager()
    a, b = _host("fully_contiguous", NHD), _host("fully_contiguous", HND)
    opts = TransferOptions()
    assert tm._pick_engine(a, b, opts, [0], [1]) == "tma"
    assert tm._pick_engine(a, b, opts, [2, 3], [4, 5]) == "tma"
    assert tm._plans.hits == 1 and tm._plans.misses == 1
    c = PreparedPlanCache(capacity=1)
    c.put(("k1",), None)
    c.put(("k2",), None)
    assert c.get(("k1",)) is None and c.misses == 1
    tm.close()
