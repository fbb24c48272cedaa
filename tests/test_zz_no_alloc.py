"""The allocation-free decode-attention entry point, called through its
exported C symbol, must match the scratch-taking entry point.

``kvbm_paged_decode_attn_noalloc`` exists for callers that cannot allocate
device memory at call time (an application that owns all device memory in
its own arena, code running inside an allocator callback, paths that cannot
absorb cudaMalloc's synchronization): its split partials live in a fixed
array inside the library. This file runs last so that, if it fails, a run
that stops at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.ops import _lib, llama_ops
from kvbm_b200.physical.layout import KvBlockLayout, KvLayout, LayoutConfig

_V, _I64, _I, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float


def _noalloc_symbol():
    lib = ctypes.CDLL(str(_lib.lib_path()))
    fn = lib.kvbm_paged_decode_attn_noalloc
    fn.restype = _I
    fn.argtypes = [_V, _V, _V, _I64, _I64, _I64, _I, _V, _I, _V, _I, _I, _I, _I, _F, _I, _V, _V]
    cap = lib.kvbm_paged_decode_attn_noalloc_max_rows
    cap.restype = _I
    msg = lib.kvbm_last_error_message
    msg.restype = ctypes.c_char_p
    return fn, cap(), msg


def _case(seed, B, hkv, group, page=16, max_seq=700):
    g = torch.Generator(device="cuda").manual_seed(seed)
    seq = torch.randint(1, max_seq, (B,), generator=g, device="cuda", dtype=torch.int32)
    max_blocks = int((int(seq.max()) + page - 1) // page)
    nb = B * max_blocks + 1
    pool = KvLayout.allocate(LayoutConfig.for_model(nb, 1, hkv, 128, page), "fully_contiguous",
                             KvBlockLayout.OPERATIONAL_NHD)
    view = pool.layer_view(0)
    view.copy_(torch.randn(view.shape, generator=g, device="cuda").to(torch.bfloat16))
    table = torch.randperm(nb - 1, generator=g, device="cuda")[: B * max_blocks].view(B, max_blocks).to(torch.int32)
    q = torch.randn(B, hkv * group, 128, generator=g, device="cuda").to(torch.bfloat16)
    return pool, table, seq, q


def test_noalloc_matches_scratch_entry_point_two_calls_in_a_row():
    fn, cap, _ = _noalloc_symbol()
    assert cap >= 1024
    scale = 1.0 / math.sqrt(128)
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row with different shapes and contents: the second must
    # not see anything left over from the first
    for seed, (B, hkv, group, splits) in enumerate([(6, 4, 4, 5), (3, 8, 2, 9)]):
        pool, table, seq, q = _case(seed, B, hkv, group)
        kb = pool.layer_base(0)
        vb = kb + pool.outer_stride
        ref = llama_ops.paged_decode_attn(q, kb, vb, pool.block_stride, pool.token_stride, pool.head_stride, 16,
                                          table, seq, hkv, scale, splits)
        out = torch.full_like(q, float("nan"))
        rc = fn(q.data_ptr(), kb, vb, pool.block_stride, pool.token_stride, pool.head_stride, 16, table.data_ptr(),
                table.shape[1], seq.data_ptr(), B, q.shape[1], hkv, 128, scale, splits, out.data_ptr(), stream)
        torch.cuda.synchronize()
        assert rc == 0
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_noalloc_rejects_requests_beyond_its_capacity():
    fn, cap, msg = _noalloc_symbol()
    pool, table, seq, q = _case(7, 2, 2, 4)
    kb = pool.layer_base(0)
    splits = cap // (2 * 8) + 1  # batch 2 x 8 query heads x splits > capacity
    out = torch.zeros_like(q)
    rc = fn(q.data_ptr(), kb, kb + pool.outer_stride, pool.block_stride, pool.token_stride, pool.head_stride, 16,
            table.data_ptr(), table.shape[1], seq.data_ptr(), 2, 8, 2, 128, 0.1, splits, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"exceeds the static scratch capacity" in msg()


def test_noalloc_at_exactly_its_capacity():
    """batch * hq * splits equal to the capacity: the partials fill the array to its last row."""
    fn, cap, msg = _noalloc_symbol()
    B, hkv, group, page = 2, 2, 4, 16
    hq = hkv * group
    splits = cap // (B * hq)
    assert B * hq * splits == cap
    seq_len = splits * page  # one block per split
    g = torch.Generator(device="cuda").manual_seed(17)
    nb = B * splits + 1
    pool = KvLayout.allocate(LayoutConfig.for_model(nb, 1, hkv, 128, page), "fully_contiguous",
                             KvBlockLayout.OPERATIONAL_NHD)
    view = pool.layer_view(0)
    view.copy_(torch.randn(view.shape, generator=g, device="cuda").to(torch.bfloat16))
    table = torch.randperm(nb - 1, generator=g, device="cuda")[: B * splits].view(B, splits).to(torch.int32)
    seq = torch.full((B,), seq_len, dtype=torch.int32, device="cuda")
    q = torch.randn(B, hq, 128, generator=g, device="cuda").to(torch.bfloat16)
    kb = pool.layer_base(0)
    vb = kb + pool.outer_stride
    scale = 1.0 / math.sqrt(128)
    ref = llama_ops.paged_decode_attn(q, kb, vb, pool.block_stride, pool.token_stride, pool.head_stride, page,
                                      table, seq, hkv, scale, splits)
    out = torch.full_like(q, float("nan"))
    rc = fn(q.data_ptr(), kb, vb, pool.block_stride, pool.token_stride, pool.head_stride, page, table.data_ptr(),
            table.shape[1], seq.data_ptr(), B, hq, hkv, 128, scale, splits, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, msg()
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
