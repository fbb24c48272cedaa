"""GPU numerics of the KV transfer kernels against PyTorch references.

Pattern (after the reference's kernel_roundtrip tests): random source blocks,
poison-filled destinations, and an exact comparison of every moved element
against a plain PyTorch gather of the same blocks; fp8 paths against an fp32
PyTorch quantiser.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.ops import _lib, kv_ops
from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig

NHD = KvBlockLayout.OPERATIONAL_NHD
HND = KvBlockLayout.OPERATIONAL_HND
UNI = KvBlockLayout.UNIVERSAL


def _cfg(nb=24, nl=4, nh=8, hd=128, page=16, dtype=torch.bfloat16):
    return LayoutConfig.for_model(nb, nl, nh, hd, page, dtype)


def _fill(lay: KvLayout, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    c = lay.config
    for l in range(c.num_layers):
        v = lay.layer_view(l)
        if lay.dtype == torch.float8_e4m3fn:
            v.view(torch.uint8).copy_(torch.randint(0, 120, v.shape, generator=g, device="cuda", dtype=torch.uint8))
        else:
            v.copy_(torch.randn(v.shape, generator=g, device="cuda", dtype=torch.float32).to(lay.dtype))


def _poison(lay: KvLayout):
    lay._flat().fill_(0x5A)


def _pairs(n, nb, seed):
    g = torch.Generator().manual_seed(seed)
    src = torch.randperm(nb, generator=g)[:n]
    dst = torch.randperm(nb, generator=g)[:n]
    return src.tolist(), dst.tolist()


@pytest.mark.parametrize("engine", ["tile", "tma"])
@pytest.mark.parametrize(
    "src_kind,src_bl,dst_kind,dst_bl,dst_block_first",
    [
        ("fully_contiguous", NHD, "fully_contiguous", NHD, True),
        ("fully_contiguous", NHD, "layer_separate", HND, True),
        ("fully_contiguous", NHD, "fully_contiguous", UNI, True),
        ("fully_contiguous", UNI, "layer_separate", NHD, False),
        ("layer_separate", HND, "fully_contiguous", NHD, True),
    ],
)
def test_layout_transfer_exact(engine, src_kind, src_bl, dst_kind, dst_bl, dst_block_first):
    cfg = _cfg()
    src = KvLayout.allocate(cfg, src_kind, src_bl)
    dst = KvLayout.allocate(cfg, dst_kind, dst_bl, block_first=dst_block_first)
    _fill(src, 1)
    _poison(dst)
    s_ids, d_ids = _pairs(10, cfg.num_blocks, 2)
    ran = kv_ops.kv_transfer(src, s_ids, dst, d_ids, engine=engine)
    same = src_kind == dst_kind == "fully_contiguous" and src_bl == dst_bl
    assert ran == ("tile" if engine == "tile" else ("tma_bulk" if same else "tma"))
    torch.cuda.synchronize()
    assert kv_ops.transfer_status(reset=True) == 0
    assert torch.equal(dst.gather_blocks(d_ids), src.gather_blocks(s_ids))
    # untouched blocks keep the poison
    others = [b for b in range(cfg.num_blocks) if b not in d_ids]
    assert bool((dst.gather_blocks(others[:3]).view(torch.uint8) == 0x5A).all())


@pytest.mark.parametrize("engine", ["tile", "tma"])
def test_layer_subrange_and_head_reshard(engine):
    # prefill TP=2 rank holds 4 of 8 heads; decode TP=1 holds all 8
    src = KvLayout.allocate(_cfg(nh=4), "fully_contiguous", NHD)
    dst = KvLayout.allocate(_cfg(nh=8), "fully_contiguous", NHD)
    _fill(src, 3)
    _poison(dst)
    s_ids, d_ids = _pairs(7, 24, 4)
    ran = kv_ops.kv_transfer(src, s_ids, dst, d_ids, layer_begin=1, num_layers=2, dst_head_offset=4, engine=engine)
    assert ran == engine  # a head slice is never a whole-chunk image: the staged pipeline, not the bulk copy
    torch.cuda.synchronize()
    got = dst.gather_blocks(d_ids)
    ref = src.gather_blocks(s_ids)
    assert torch.equal(got[:, 1:3, :, :, 4:8], ref[:, 1:3])
    assert bool((got[:, 0].view(torch.uint8) == 0x5A).all())
    assert bool((got[:, 1:3, :, :, 0:4].contiguous().view(torch.uint8) == 0x5A).all())


def _ref_quant(x: torch.Tensor):
    """x: [..., page, heads, hd] per (block, layer, outer) -> per-head scales over (page, hd)."""
    xf = x.float()
    amax = xf.abs().amax(dim=(-3, -1))  # [..., heads]
    # tensor / tensor divisions round correctly (torch computes a division by a scalar, or of a scalar, as a
    # multiplication by a reciprocal, which can differ in the last bit from the kernel's fp32 division)
    c448 = torch.full_like(amax, 448.0)
    scale = torch.where(amax > 0, amax / c448, torch.ones_like(amax))
    inv = torch.where(amax > 0, c448 / amax, torch.ones_like(amax))
    q = (xf * inv.unsqueeze(-2).unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q, scale


@pytest.mark.parametrize("engine", ["tile", "tile_sw1", "tile_sw", "tile1", "tma"])
@pytest.mark.parametrize("src_dtype", [torch.bfloat16, torch.float16])
def test_fp8_quant_dequant(engine, src_dtype):
    # tile: the software-pipelined cast kernel; tile_sw: the same with the conversions on the
    # integer / FMA pipes; tile1: the one-tile-at-a-time kernel
    kv_ops.set_cast_pipeline(engine != "tile1")
    sq = {"tile_sw1": 1, "tile_sw": 4}.get(engine, 0)
    kv_ops.set_cast_softconv(sq, sq)
    try:
        _fp8_roundtrip("tile" if engine.startswith("tile") else engine, src_dtype)
    finally:
        kv_ops.set_cast_pipeline(True)
        kv_ops.set_cast_softconv()


def _fp8_roundtrip(engine, src_dtype):
    cfg = _cfg(dtype=src_dtype)
    cfg8 = _cfg(dtype=torch.float8_e4m3fn)
    src = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    q8 = KvLayout.allocate(cfg8, "fully_contiguous", HND, fp8_scales=True)
    back = KvLayout.allocate(cfg, "layer_separate", NHD)
    _fill(src, 5)
    s_ids, d_ids = _pairs(9, 24, 6)
    assert kv_ops.kv_transfer(src, s_ids, q8, d_ids, engine=engine) == engine
    assert kv_ops.kv_transfer(q8, d_ids, back, s_ids, engine=engine) == engine
    torch.cuda.synchronize()
    x = src.gather_blocks(s_ids)  # [n, L, O, T, H, D]
    qref, sref = _ref_quant(x)
    got_q = q8.gather_blocks(d_ids).view(torch.float8_e4m3fn)
    got_s = q8.scales_view()[torch.tensor(d_ids, device="cuda")]
    assert torch.equal(got_s, sref)
    # same fp32 scale, same fp32 product, both round to nearest even with saturation: byte-exact
    mism = (got_q.view(torch.uint8) != qref.view(torch.uint8))
    assert int(mism.sum()) == 0, (int(mism.sum()), x[mism].flatten()[:8].tolist())
    deq = back.gather_blocks(s_ids).float()
    # the dequantiser is exact given the stored fp8 bytes and scales
    ref_deq = (got_q.float() * got_s.unsqueeze(-2).unsqueeze(-1)).to(src_dtype).float()
    bad = (deq != ref_deq).float().mean().item()
    assert bad == 0.0, bad
    err = (deq - x.float()).abs()
    bound = 0.0625 * x.float().abs() + sref.unsqueeze(-2).unsqueeze(-1) * 2.0 ** -9 + 1e-2 * x.float().abs()
    assert bool((err <= bound).all())


def test_fp8_copy_carries_scales():
    cfg8 = _cfg(dtype=torch.float8_e4m3fn)
    a = KvLayout.allocate(cfg8, "fully_contiguous", NHD, fp8_scales=True)
    b = KvLayout.allocate(cfg8, "layer_separate", HND, fp8_scales=True)
    _fill(a, 7)
    a.scales_view().copy_(torch.rand_like(a.scales_view()))
    s_ids, d_ids = _pairs(5, 24, 8)
    kv_ops.kv_transfer(a, s_ids, b, d_ids)
    torch.cuda.synchronize()
    assert torch.equal(b.gather_blocks(d_ids).view(torch.uint8), a.gather_blocks(s_ids).view(torch.uint8))
    assert torch.equal(b.scales_view()[torch.tensor(d_ids, device="cuda")],
                       a.scales_view()[torch.tensor(s_ids, device="cuda")])


def test_transfer_to_pinned_host_and_back():
    cfg = _cfg()
    g1 = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    g2 = KvLayout.allocate(cfg, "fully_contiguous", NHD, location="pinned")
    g1b = KvLayout.allocate(cfg, "layer_separate", NHD)
    _fill(g1, 9)
    s_ids, d_ids = _pairs(12, 24, 10)
    kv_ops.kv_transfer(g1, s_ids, g2, d_ids)  # offload G1 -> G2 by SM kernel
    kv_ops.kv_transfer(g2, d_ids, g1b, s_ids)  # onboard G2 -> G1
    torch.cuda.synchronize()
    assert torch.equal(g2.gather_blocks(d_ids).cuda(), g1.gather_blocks(s_ids))
    assert torch.equal(g1b.gather_blocks(s_ids), g1.gather_blocks(s_ids))


@pytest.mark.parametrize("hugepages", [False, True])
def test_transfer_through_numa_placed_pool(hugepages):
    # G2 on the GPU's NUMA node (huge pages when the host has them), page-locked and mapped
    cfg = _cfg()
    g1 = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    g2 = KvLayout.allocate(cfg, "fully_contiguous", NHD, location="pinned", numa_node="gpu", hugepages=hugepages)
    assert g2.backing.pinned and g2.backing.device_ptr
    g1b = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    _fill(g1, 4)
    s_ids, d_ids = _pairs(12, 24, 10)
    kv_ops.kv_transfer(g1, s_ids, g2, d_ids)
    kv_ops.kv_transfer(g2, d_ids, g1b, s_ids)
    torch.cuda.synchronize()
    assert torch.equal(g1b.gather_blocks(s_ids), g1.gather_blocks(s_ids))


@pytest.mark.parametrize("nbytes", [1, 7, 16, 4096, 65536 + 48, 2 << 20])
def test_copy_pairs(nbytes):
    n = 6
    src = torch.randint(0, 255, (n, nbytes + 64), dtype=torch.uint8, device="cuda")
    dst = torch.zeros((n, nbytes + 64), dtype=torch.uint8, device="cuda")
    off = 3 if nbytes % 16 else 0
    sp = [src[i].data_ptr() + off for i in range(n)]
    dp = [dst[i].data_ptr() + off for i in range(n)]
    kv_ops.copy_pairs(sp, dp, nbytes)
    torch.cuda.synchronize()
    assert torch.equal(dst[:, off:off + nbytes], src[:, off:off + nbytes])
    assert int(dst[:, :off].sum()) == 0 and int(dst[:, off + nbytes:].sum()) == 0


def test_copy_pairs_empty_is_noop():
    kv_ops.copy_pairs([], [], 0)


def _chunk_table(chunks):
    return torch.tensor([c.data_ptr() for c in chunks], dtype=torch.int64, device="cuda")


@pytest.mark.parametrize("layout", [_lib.NHD, _lib.HND])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float64, torch.float8_e4m3fn])
def test_reference_compatible_permutes(layout, dtype):
    nb, nh, nl, no, nt, hd = 3, 4, 3, 2, 16, 64
    nl_full, nl_off = 5, 2
    gen = torch.Generator(device="cuda").manual_seed(11)
    store = torch.float32 if dtype == torch.float8_e4m3fn else dtype

    def rnd(shape):
        x = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).to(store)
        return x.to(dtype) if dtype == torch.float8_e4m3fn else x

    inner = (nt, nh, hd) if layout == _lib.NHD else (nh, nt, hd)
    chunks = [rnd(inner) for _ in range(nb * nl * no)]
    univ = [torch.zeros((nh, nl_full, no, nt, hd), dtype=dtype, device="cuda") for _ in range(nb)]
    uptr = _chunk_table(univ)
    bptr = _chunk_table(chunks)
    kv_ops.universal_from_block(uptr, bptr, nh, nl, no, nt, hd, dtype, layout, nl_full=nl_full, nl_offset=nl_off)
    torch.cuda.synchronize()
    u8 = (lambda z: z.view(torch.uint8)) if dtype == torch.float8_e4m3fn else (lambda z: z)
    for b in range(nb):
        for l in range(nl):
            for o in range(no):
                c = u8(chunks[(b * nl + l) * no + o])
                c_nhd = c if layout == _lib.NHD else c.transpose(0, 1)
                got = u8(univ[b])[:, nl_off + l, o].transpose(0, 1)  # [nt, nh, hd]
                assert torch.equal(got, c_nhd)
    back = [torch.zeros_like(c) for c in chunks]
    kv_ops.block_from_universal(uptr, _chunk_table(back), nh, nl, no, nt, hd, dtype, layout, nl_full=nl_full,
                                nl_offset=nl_off)
    trans = [torch.zeros((inner[1], inner[0], hd), dtype=dtype, device="cuda") for _ in chunks]
    kv_ops.nhd_hnd_transpose(bptr, _chunk_table(trans), nb, nl, no, nt, nh, hd, dtype, layout)
    torch.cuda.synchronize()
    u8 = (lambda z: z.view(torch.uint8)) if dtype == torch.float8_e4m3fn else (lambda z: z)
    for c, r, t in zip(chunks, back, trans):
        assert torch.equal(u8(c), u8(r))
        assert torch.equal(u8(c).transpose(0, 1).contiguous(), u8(t))


def test_permute_rejects_bad_layer_range():
    t = torch.zeros(4, dtype=torch.int64, device="cuda")
    with pytest.raises(_lib.KvbmCudaError):
        kv_ops.universal_from_block(t[:1], t, 2, 3, 2, 16, 64, torch.bfloat16, _lib.NHD, nl_full=2, nl_offset=0)


def test_flag_signal_wait_and_timeout():
    flag = torch.zeros(2, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kv_ops.signal_flag(flag.data_ptr(), 5)
    kv_ops.wait_flag(flag.data_ptr(), 5, 1_000_000_000, status.data_ptr())
    torch.cuda.synchronize()
    assert int(flag[0]) == 5 and int(status[0]) == 0
    # nothing sets flag[1]: the bounded wait gives up and reports a timeout
    kv_ops.wait_flag(flag.data_ptr() + 8, 1, 2_000_000, status.data_ptr())
    torch.cuda.synchronize()
    assert int(status[0]) == 1
    # the context stays usable
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_checksum_kernel_matches_reference_across_layouts(dtype):
    from kvbm_b200.physical.verify import FillPattern, checksum_blocks, checksum_reference, fill_blocks

    cfg = LayoutConfig.for_model(10, 3, 4, 128, 16, dtype)
    a = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, zero=True)
    b = KvLayout.allocate(cfg, "layer_separate", KvBlockLayout.OPERATIONAL_HND, zero=True)
    h = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_HND, location="pinned", zero=True)
    fill_blocks(a, [1, 4, 7], FillPattern.RANDOM, seed=5)
    kv_ops.kv_transfer(a, [1, 4, 7], b, [0, 2, 9])
    kv_ops.kv_transfer(a, [1, 4, 7], h, [3, 5, 6])
    torch.cuda.synchronize()
    ca = checksum_blocks(a, [1, 4, 7])
    assert ca == checksum_blocks(b, [0, 2, 9]) == checksum_blocks(h, [3, 5, 6])
    assert ca == [checksum_reference(x) for x in a.gather_blocks([1, 4, 7])]
    assert len(set(ca)) == 3
    sub = checksum_blocks(b, [2], layer_begin=1, num_layers=2)
    assert sub == [checksum_reference(a.gather_blocks([4])[0, 1:3])]


@pytest.mark.parametrize("nh", [1, 2, 3, 8])
@pytest.mark.parametrize("fp8", [False, True])
def test_tma_head_slices_match_tile_engine(nh, fp8):
    """Head slices narrower than the TMA pipeline's 8 consumer warps (a TP rank's
    share): grouped consumers must store exactly what the tile engine stores."""
    src_cfg = _cfg(nb=20, nl=3, nh=nh)
    dst_cfg = _cfg(nb=20, nl=3, nh=2 * nh, dtype=torch.float8_e4m3fn if fp8 else torch.bfloat16)
    src = KvLayout.allocate(src_cfg, "fully_contiguous", NHD)
    _fill(src, 11)
    s_ids, d_ids = _pairs(13, 20, 12)
    outs = []
    for engine in ("tile", "tma"):
        dst = KvLayout.allocate(dst_cfg, "fully_contiguous", HND, fp8_scales=fp8)
        _poison(dst)
        kv_ops.kv_transfer(src, s_ids, dst, d_ids, dst_head_offset=nh, num_heads=nh, engine=engine)
        torch.cuda.synchronize()
        got = dst.gather_blocks(d_ids).view(torch.uint8)
        outs.append((got, dst.scales_view()[torch.tensor(d_ids, device="cuda")].clone() if fp8 else None))
    assert torch.equal(outs[0][0], outs[1][0])
    if fp8:
        assert torch.equal(outs[0][1][..., nh:], outs[1][1][..., nh:])
    else:
        ref = src.gather_blocks(s_ids)
        assert torch.equal(outs[1][0].view(torch.bfloat16)[..., nh:, :], ref.view(torch.bfloat16))


def test_bulk_copy_many_chunks_exact_and_opt_out():
    """Same-layout copies go through the TMA bulk copy (loads and stores by the TMA unit);
    more chunks than CTAs x stages exercises the stage refill; bulk=False keeps the pipeline."""
    cfg = _cfg(nb=300, nl=4)
    src = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    _fill(src, 21)
    s_ids, d_ids = _pairs(290, 300, 22)
    for bulk, want in ((None, "tma_bulk"), (False, "tma")):
        dst = KvLayout.allocate(cfg, "fully_contiguous", NHD)
        _poison(dst)
        assert kv_ops.kv_transfer(src, s_ids, dst, d_ids, engine="tma", bulk=bulk) == want
        torch.cuda.synchronize()
        assert kv_ops.transfer_status(reset=True) == 0
        assert torch.equal(dst.gather_blocks(d_ids), src.gather_blocks(s_ids))
    # a layer sub-range is still a whole-chunk image per (block, layer, outer)
    dst = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    _poison(dst)
    assert kv_ops.kv_transfer(src, s_ids, dst, d_ids, layer_begin=1, num_layers=2, engine="tma") == "tma_bulk"
    torch.cuda.synchronize()
    assert torch.equal(dst.gather_blocks(d_ids)[:, 1:3], src.gather_blocks(s_ids)[:, 1:3])
    assert bool((dst.gather_blocks(d_ids)[:, 0].view(torch.uint8) == 0x5A).all())


def test_tma_rejects_instead_of_falling_back():
    """engine='tma' on a source whose chunks are neither token- nor head-contiguous raises;
    'auto' runs the tile kernel."""
    base = _cfg(nb=8, nl=2, nh=8)
    src = KvLayout.allocate(base, "fully_contiguous", NHD)
    _fill(src, 41)
    # every other head of the pool: rows of one token are 2 rows apart, tokens 8 rows apart
    half = _cfg(nb=8, nl=2, nh=4)
    strided = KvLayout(half, "fully_contiguous", NHD, src.base_ptr, src.layer_offsets, src.block_stride,
                       src.outer_stride, src.token_stride, src.head_stride * 2, src.nbytes, "device", src.device, src)
    dst = KvLayout.allocate(half, "fully_contiguous", NHD)
    with pytest.raises(_lib.KvbmCudaError):
        kv_ops.kv_transfer(strided, [0, 1], dst, [2, 3], engine="tma")
    assert kv_ops.kv_transfer(strided, [0, 1], dst, [2, 3], engine="auto") == "tile"
    torch.cuda.synchronize()
    assert torch.equal(dst.gather_blocks([2, 3]), src.gather_blocks([0, 1])[..., 0::2, :])


@pytest.mark.parametrize("bulk", [None, False])
def test_pipeline_timeout_reports_status_without_fault(bulk):
    """A pipeline wait with a 1 ns limit gives up: the kernel drains the copies it issued,
    returns, and the host reads status 3; the next transfer with the normal limit is exact."""
    cfg = _cfg(nb=64, nl=4)
    src = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    dst = KvLayout.allocate(cfg, "fully_contiguous", NHD)
    _fill(src, 31)
    s_ids, d_ids = _pairs(60, 64, 32)
    kv_ops.transfer_status(reset=True)
    kv_ops.set_pipeline_wait_limit_ns(1)
    try:
        kv_ops.kv_transfer(src, s_ids, dst, d_ids, engine="tma", bulk=bulk)
        torch.cuda.synchronize()
    finally:
        kv_ops.set_pipeline_wait_limit_ns(0)
    assert kv_ops.transfer_status() == 3
    with pytest.raises(_lib.KvbmCudaError):
        kv_ops.check_transfer_status()
    assert kv_ops.transfer_status() == 0  # check_transfer_status cleared it
    _poison(dst)
    kv_ops.kv_transfer(src, s_ids, dst, d_ids, engine="tma", bulk=bulk)
    torch.cuda.synchronize()
    kv_ops.check_transfer_status()
    assert torch.equal(dst.gather_blocks(d_ids), src.gather_blocks(s_ids))


@pytest.mark.parametrize("layout", ["NHD", "HND"])
@pytest.mark.parametrize("backend", [None, "async"])
def test_tensor_level_kernels_api(layout, backend):
    """``kvbm.kernels``: block stacks <-> universal tensors and <-> operational buffers, checked
    exactly against PyTorch permutes / concatenation of the same tensors."""
    from kvbm import kernels

    nb, nh, nl, no, nt, hd = 2, 4, 3, 2, 16, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    inner = (nt, nh, hd) if layout == "NHD" else (nh, nt, hd)
    blocks = [[torch.randn(inner, generator=g, device="cuda").to(torch.bfloat16) for _ in range(nl * no)]
              for _ in range(nb)]
    unis = [torch.zeros((nh, nl, no, nt, hd), dtype=torch.bfloat16, device="cuda") for _ in range(nb)]
    kernels.block_to_universal(blocks, unis, layout)
    for b in range(nb):
        for l in range(nl):
            for o in range(no):
                c = blocks[b][l * no + o]
                want = c.transpose(0, 1) if layout == "NHD" else c  # [nh, nt, hd]
                assert torch.equal(unis[b][:, l, o], want)
    back = [[torch.zeros_like(c) for c in grp] for grp in blocks]
    kernels.universal_to_block(unis, back, layout)
    assert all(torch.equal(x, y) for gx, gy in zip(blocks, back) for x, y in zip(gx, gy))
    ops = [torch.zeros((nl, no, nt * nh * hd), dtype=torch.bfloat16, device="cuda") for _ in range(nb)]
    kernels.block_to_operational(blocks, ops, backend=backend)
    for b in range(nb):
        assert torch.equal(ops[b].reshape(-1), torch.cat([c.reshape(-1) for c in blocks[b]]))
    back2 = [[torch.zeros_like(c) for c in grp] for grp in blocks]
    kernels.operational_to_block(ops, back2, backend=backend)
    assert all(torch.equal(x, y) for gx, gy in zip(blocks, back2) for x, y in zip(gx, gy))
    one = torch.zeros((nh, nl, no, nt, hd), dtype=torch.bfloat16, device="cuda")
    kernels.block_to_universal(blocks[0], one, layout)  # a single universal tensor is one block
    assert torch.equal(one, unis[0])
