"""CPU tests: labelled KV tensor algebra (axes, strides, slices, intersections)."""

import pytest
import torch

from kvbm_b200.common.tensor import (AxisExtent, AxisSlice, CanonicalBlockShape, CoordByLabel, KvbmTransferRoute,
                                     KvDim, KvDimLayout, KvDimStrides, LayoutSignature, LogicalLayoutHandle,
                                     intersect_axis)
from kvbm_b200.parallel.tp import ParallelismTemplate, plan_pull

D = KvDim


def test_layout_invariants():
    lay = KvDimLayout([D.BLOCK, D.OUTER, D.PAGE, D.HEAD, D.HEAD_SIZE], [10, 2, 16, 8, 128])
    assert lay.block_axis == 0 and lay.outer_size == 2 and lay.page_size == 16
    assert lay.inner_elements == 16 * 8 * 128 and lay.inner_bytes(2) == 32768
    assert lay.total_elements == 10 * 2 * 16 * 8 * 128
    for dims, sizes in [([D.PAGE, D.HEAD_SIZE], [16, 128]),                       # no block axis
                        ([D.BLOCK, D.BLOCK, D.HEAD_SIZE], [2, 2, 8]),             # two block axes
                        ([D.BLOCK, D.OUTER, D.HEAD_SIZE], [4, 3, 8]),             # outer of 3
                        ([D.BLOCK, D.PAYLOAD, D.PAGE], [4, 8, 16]),               # payload not last
                        ([D.BLOCK, D.HEAD_SIZE, D.PAYLOAD], [4, 8, 16]),          # both tails
                        ([D.BLOCK, D.PAGE], [4, 0])]:                             # zero size
        with pytest.raises(ValueError):
            KvDimLayout(dims, sizes)


def test_strides_match_torch_and_contiguous_tail():
    lay = KvDimLayout([D.OUTER, D.BLOCK, D.PAGE, D.HEAD, D.HEAD_SIZE], [2, 6, 16, 4, 64])
    t = torch.empty(lay.sizes, dtype=torch.bfloat16)
    st = KvDimStrides.from_element_strides(t.stride(), 2)
    assert st == KvDimStrides.contiguous_for(lay, 2) and st.is_fully_contiguous(lay)
    # a per-block view that skips the other half of outer: the tail below OUTER is one run
    half = t[0:1]
    assert KvDimStrides.from_element_strides(half.stride(), 2).contiguous_tail_bytes(
        KvDimLayout(lay.dims, half.shape)) == 6 * 16 * 4 * 64 * 2
    # HND permuted view: only head_size is contiguous
    perm = t.permute(0, 1, 3, 2, 4)
    lay2 = KvDimLayout([D.OUTER, D.BLOCK, D.HEAD, D.PAGE, D.HEAD_SIZE], perm.shape)
    assert KvDimStrides.from_element_strides(perm.stride(), 2).contiguous_tail_bytes(lay2) == 128
    with pytest.raises(ValueError):
        KvDimStrides.from_byte_strides([3, 1], 2)
    c = CoordByLabel().with_(D.BLOCK, 2).with_(D.HEAD, 1)
    assert c.offset(lay, st) == 2 * st.byte_strides[1] + 1 * st.byte_strides[3]
    with pytest.raises(IndexError):
        CoordByLabel().with_(D.OUTER, 2).offset(lay, st)


def test_slices_and_intersections():
    s = AxisSlice.full(D.HEAD, 32)
    assert s.is_full and s.end == 32
    shards = [AxisSlice.shard(D.HEAD, r, 4, 32) for r in range(4)]
    assert [(x.start, x.len) for x in shards] == [(0, 8), (8, 8), (16, 8), (24, 8)]
    with pytest.raises(ValueError):
        AxisSlice.shard(D.HEAD, 0, 3, 32)
    with pytest.raises(ValueError):
        AxisSlice.shard(D.HEAD, 4, 4, 32)
    with pytest.raises(ValueError):
        AxisSlice(D.HEAD, 24, 16, 32)
    inter = intersect_axis(s, shards[1])
    assert inter.src_local == range(8, 16) and inter.dst_local == range(0, 8) and len(inter) == 8
    assert intersect_axis(shards[0], shards[1]) is None
    wide = AxisSlice.shard(D.HEAD, 1, 2, 32)  # [16, 32)
    i2 = intersect_axis(shards[3], wide)
    assert i2.src_local == range(0, 8) and i2.dst_local == range(8, 16)
    with pytest.raises(ValueError):
        intersect_axis(s, AxisSlice.full(D.LAYER, 32))
    with pytest.raises(ValueError):
        intersect_axis(s, AxisSlice.full(D.HEAD, 16))
    assert AxisExtent.from_slice(wide) == AxisExtent(16, 32, 16) and AxisExtent.full(4).is_full


@pytest.mark.parametrize("lt,rt", [(1, 1), (2, 2), (1, 8), (2, 8), (8, 2), (8, 1), (4, 2)])
def test_plan_pull_covers_every_head_once(lt, rt):
    G = 8
    plans = plan_pull(ParallelismTemplate(lt, G, 4), ParallelismTemplate(rt, G, 4))
    for p in plans:
        got = []
        for sh in p.shards:
            lo = p.local_rank * (G // lt) + sh.local_head_offset
            rlo = sh.remote_rank * (G // rt) + sh.remote_head_offset
            assert lo == rlo  # the same global heads on both sides
            got.extend(range(lo, lo + sh.num_heads))
        assert got == list(range(p.local_rank * (G // lt), (p.local_rank + 1) * (G // lt)))


def test_signature_routes_and_shapes():
    a = LayoutSignature(((D.BLOCK, AxisExtent.full(8)), (D.HEAD, AxisExtent(4, 8, 0))), (4096, 512), 2)
    b = LayoutSignature(((D.BLOCK, AxisExtent.full(8)), (D.HEAD, AxisExtent(2, 8, 6))), (2048, 256), 2)
    assert a.compatible(b)
    assert not a.compatible(LayoutSignature(((D.BLOCK, AxisExtent.full(8)),), (4096,), 2))
    G = LogicalLayoutHandle
    assert KvbmTransferRoute.of(G.G1, G.G2) == KvbmTransferRoute.OFFLOAD_D2H
    assert KvbmTransferRoute.of(G.G3, G.G2) == KvbmTransferRoute.ONBOARD_D2H
    with pytest.raises(ValueError):
        KvbmTransferRoute.of(G.G1, G.G1)
    x = CanonicalBlockShape(32, 2, 16, 8, 128, 2)
    x.require_equal(CanonicalBlockShape(32, 2, 16, 8, 128, 2))
    with pytest.raises(ValueError, match="num_heads"):
        x.require_equal(CanonicalBlockShape(32, 2, 16, 4, 128, 2))
