"""GPU numerics of the fused Llama ops against plain PyTorch fp32 references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.ops import llama_ops
from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig


def test_rmsnorm_with_residual():
    torch.manual_seed(0)
    x = torch.randn(37, 4096, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(37, 4096, device="cuda", dtype=torch.bfloat16)
    w = torch.rand(4096, device="cuda", dtype=torch.bfloat16) + 0.5
    r_ref = (x.float() + r.float()).to(torch.bfloat16)
    var = r_ref.float().pow(2).mean(-1, keepdim=True)
    ref = (r_ref.float() * torch.rsqrt(var + 1e-5)).to(torch.bfloat16).float() * w.float()
    r2 = r.clone()
    out = llama_ops.rmsnorm(x, w, 1e-5, residual=r2)
    torch.cuda.synchronize()
    assert torch.equal(r2, r_ref)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)
    out2 = llama_ops.rmsnorm(x, w, 1e-5)
    var = x.float().pow(2).mean(-1, keepdim=True)
    ref2 = (x.float() * torch.rsqrt(var + 1e-5)).to(torch.bfloat16).float() * w.float()
    torch.testing.assert_close(out2.float(), ref2, rtol=1e-2, atol=1e-2)


def _cos_sin(max_pos, hd, theta=500000.0):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    f = torch.outer(torch.arange(max_pos, dtype=torch.float64), inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).float().cuda()


def _rope_ref(x, pos, cs):
    hd = x.shape[-1]
    c = cs[pos][:, None, : hd // 2]
    s = cs[pos][:, None, hd // 2:]
    x1, x2 = x[..., : hd // 2].float(), x[..., hd // 2:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def test_rope_kv_write_paged():
    torch.manual_seed(1)
    T, hq, hkv, hd, page = 50, 32, 8, 128, 16
    cfg = LayoutConfig.for_model(16, 2, hkv, hd, page)
    pool = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, zero=True)
    qkv = torch.randn(T, hq + 2 * hkv, hd, device="cuda", dtype=torch.bfloat16)
    orig = qkv.clone()
    pos = torch.arange(100, 100 + T, device="cuda", dtype=torch.int32)
    cs = _cos_sin(4096, hd)
    blocks = torch.tensor([5, 2, 9, 11], device="cuda")
    slots = (blocks[torch.arange(T, device="cuda") // page] * page + torch.arange(T, device="cuda") % page).long()
    layer = 1
    kb = pool.layer_base(layer)
    vb = kb + pool.outer_stride
    llama_ops.rope_kv_write(qkv, pos, cs, hq, hkv, hd, kb, vb, pool.block_stride, pool.token_stride,
                            pool.head_stride, page, slots)
    torch.cuda.synchronize()
    q_ref = _rope_ref(orig[:, :hq], pos.long(), cs)
    k_ref = _rope_ref(orig[:, hq:hq + hkv], pos.long(), cs)
    torch.testing.assert_close(qkv[:, :hq].float(), q_ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(qkv[:, hq:hq + hkv].float(), k_ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(qkv[:, hq + hkv:], orig[:, hq + hkv:])
    view = pool.layer_view(layer)  # [blocks, outer, page, heads, hd]
    for t in range(T):
        b, o = int(blocks[t // page]), t % page
        assert torch.equal(view[b, 0, o], qkv[t, hq:hq + hkv])
        assert torch.equal(view[b, 1, o], orig[t, hq + hkv:])


@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("local_write", [False, True])
def test_rope_kv_push_into_second_pool(local_write, split):
    """The fused kernel rotates q/k in place and stores K/V into a second
    (HND, wider-headed) pool at a head offset, optionally also the local one."""
    torch.manual_seed(3)
    T, hq, hkv, hd, page = 70, 32, 4, 128, 16
    local = KvLayout.allocate(LayoutConfig.for_model(8, 2, hkv, hd, page), "fully_contiguous",
                              KvBlockLayout.OPERATIONAL_NHD, zero=True)
    remote = KvLayout.allocate(LayoutConfig.for_model(12, 2, 2 * hkv, hd, page), "fully_contiguous",
                               KvBlockLayout.OPERATIONAL_HND, zero=True)
    qkv = torch.randn(T, hq + 2 * hkv, hd, device="cuda", dtype=torch.bfloat16)
    orig = qkv.clone()
    pos = torch.arange(7, 7 + T, device="cuda", dtype=torch.int32)
    cs = _cos_sin(4096, hd)
    lblocks = torch.tensor([1, 0, 6, 3, 2], device="cuda")
    rblocks = torch.tensor([10, 4, 0, 7, 11], device="cuda")
    ar = torch.arange(T, device="cuda")
    lslots = (lblocks[ar // page] * page + ar % page).long()
    rslots = (rblocks[ar // page] * page + ar % page).long()
    rslots[3] = -1  # a skipped token
    layer = 1
    lk = local.layer_base(layer)
    rk = remote.layer_base(layer)
    llama_ops.rope_kv_push(qkv, pos, cs, hq, hkv,
                           (lk, lk + local.outer_stride, local.block_stride, local.token_stride, local.head_stride,
                            page, lslots) if local_write else None,
                           (rk, rk + remote.outer_stride, remote.block_stride, remote.token_stride,
                            remote.head_stride, page, rslots), r_head_offset=hkv, heads="kv" if split else "all")
    if split:
        assert torch.equal(qkv[:, :hq], orig[:, :hq])  # the K/V launch leaves the query heads alone
        llama_ops.rope_kv_push(qkv, pos, cs, hq, hkv, None, None, heads="q")
    torch.cuda.synchronize()
    q_ref = _rope_ref(orig[:, :hq], pos.long(), cs)
    k_ref = _rope_ref(orig[:, hq:hq + hkv], pos.long(), cs)
    torch.testing.assert_close(qkv[:, :hq].float(), q_ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(qkv[:, hq:hq + hkv].float(), k_ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(qkv[:, hq + hkv:], orig[:, hq + hkv:])
    rv = remote.layer_view(layer)  # [blocks, outer, page, heads, hd] whatever the physical order
    lv = local.layer_view(layer)
    for t in range(T):
        b, o = int(rblocks[t // page]), t % page
        if t == 3:
            assert not rv[b, :, o].any()
        else:
            assert not rv[b, :, o, :hkv].any()  # heads below the offset untouched
            assert torch.equal(rv[b, 0, o, hkv:], qkv[t, hq:hq + hkv])
            assert torch.equal(rv[b, 1, o, hkv:], orig[t, hq + hkv:])
        lb = int(lblocks[t // page])
        if local_write:
            assert torch.equal(lv[lb, 0, o], qkv[t, hq:hq + hkv])
            assert torch.equal(lv[lb, 1, o], orig[t, hq + hkv:])
    if not local_write:
        assert not lv.any()


def test_rope_kv_write_qout_decode_form():
    torch.manual_seed(5)
    T, hq, hkv, hd, page = 33, 32, 8, 128, 16
    cfg = LayoutConfig.for_model(8, 1, hkv, hd, page)
    pool = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD, zero=True)
    qkv = torch.randn(T, hq + 2 * hkv, hd, device="cuda", dtype=torch.bfloat16)
    orig = qkv.clone()
    pos = torch.randint(0, 4000, (T,), device="cuda", dtype=torch.int32)
    cs = _cos_sin(4096, hd)
    slots = torch.randperm(8 * page, device="cuda")[:T].long()
    q_out = torch.empty(T, hq, hd, device="cuda", dtype=torch.bfloat16)
    kb = pool.layer_base(0)
    llama_ops.rope_kv_write_qout(qkv, pos, cs, hq, hkv, kb, kb + pool.outer_stride, pool.block_stride,
                                 pool.token_stride, pool.head_stride, page, slots, q_out)
    torch.cuda.synchronize()
    torch.testing.assert_close(q_out.float(), _rope_ref(orig[:, :hq], pos.long(), cs), rtol=1e-2, atol=1e-2)
    assert torch.equal(qkv[:, :hq], orig[:, :hq])  # the q slice of qkv is left alone
    view = pool.layer_view(0)
    for t in range(T):
        b, o = int(slots[t]) // page, int(slots[t]) % page
        assert torch.equal(view[b, 0, o], qkv[t, hq:hq + hkv])
        assert torch.equal(view[b, 1, o], orig[t, hq + hkv:])


def test_silu_mul():
    torch.manual_seed(2)
    gu = torch.randn(33, 2 * 1024, device="cuda", dtype=torch.bfloat16)
    out = llama_ops.silu_mul(gu)
    g, u = gu[:, :1024].float(), gu[:, 1024:].float()
    ref = torch.nn.functional.silu(g).to(torch.bfloat16).float() * u
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("impl", ["mma", "simt", "mma_fused"])
@pytest.mark.parametrize("group", [1, 4, 8])
@pytest.mark.parametrize("splits", [1, 3, 8])
def test_paged_decode_attention(group, splits, impl):
    torch.manual_seed(3)
    B, hkv, hd, page = 5, 2, 128, 16
    hq = hkv * group
    seq = torch.tensor([1, 17, 64, 100, 333], dtype=torch.int32, device="cuda")
    max_blocks = int((seq.max() + page - 1) // page)
    nb = B * max_blocks + 3
    cfg = LayoutConfig.for_model(nb, 1, hkv, hd, page)
    pool = KvLayout.allocate(cfg, "fully_contiguous", KvBlockLayout.OPERATIONAL_NHD)
    pool.layer_view(0).copy_(torch.randn(pool.layer_view(0).shape, device="cuda").to(torch.bfloat16))
    perm = torch.randperm(nb, device="cuda")[: B * max_blocks].view(B, max_blocks).to(torch.int32)
    q = torch.randn(B, hq, hd, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(hd)
    kb = pool.layer_base(0)
    counters = torch.zeros(B * hkv, dtype=torch.int32, device="cuda") if impl == "mma_fused" else None
    kind = "mma" if impl == "mma_fused" else impl
    out = llama_ops.paged_decode_attn(q, kb, kb + pool.outer_stride, pool.block_stride, pool.token_stride,
                                      pool.head_stride, page, perm, seq, hkv, scale, splits, impl=kind,
                                      counters=counters)
    if counters is not None:
        # the tickets are re-armed: a second launch on the same buffer gives the same answer
        again = llama_ops.paged_decode_attn(q, kb, kb + pool.outer_stride, pool.block_stride, pool.token_stride,
                                            pool.head_stride, page, perm, seq, hkv, scale, splits, impl=kind,
                                            counters=counters)
        torch.cuda.synchronize()
        assert not counters.any() and torch.equal(again, out)
    torch.cuda.synchronize()
    view = pool.layer_view(0)
    for b in range(B):
        n = int(seq[b])
        blks = perm[b, : (n + page - 1) // page].long()
        k = view[blks, 0].reshape(-1, hkv, hd)[:n].float()  # [n, hkv, hd]
        v = view[blks, 1].reshape(-1, hkv, hd)[:n].float()
        qq = q[b].float().view(hkv, group, hd)
        s = torch.einsum("hgd,nhd->hgn", qq, k) * scale
        p = torch.softmax(s, dim=-1)
        ref = torch.einsum("hgn,nhd->hgd", p, v).reshape(hq, hd)
        torch.testing.assert_close(out[b].float(), ref, rtol=2e-2, atol=2e-2)
