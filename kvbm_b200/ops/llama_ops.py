"""Python entry points of the fused Llama ops (sm_100a, libkvbm_cuda.so)."""

from __future__ import annotations

import math

import torch

from . import _lib
from .kv_ops import _stream


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """out = rmsnorm(x [+ residual]) * weight; updates ``residual`` in place when given."""
    assert x.dtype == torch.bfloat16 and x.is_contiguous()
    D = x.shape[-1]
    rows = x.numel() // D
    if out is None:
        out = torch.empty_like(x)
    _lib.call("kvbm_rmsnorm", x.data_ptr(), residual.data_ptr() if residual is not None else None,
              weight.data_ptr(), out.data_ptr(), rows, D, float(eps), _stream(stream))
    return out


def rope_kv_write(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, hq: int, hkv: int, hd: int,
                  k_base: int = 0, v_base: int = 0, block_stride: int = 0, token_stride: int = 0,
                  head_stride: int = 0, page: int = 16, slots: torch.Tensor | None = None, stream=None) -> None:
    """In-place RoPE on the q/k heads of ``qkv`` [T, hq+2*hkv, hd]; writes k/v into the paged cache."""
    T = qkv.shape[0]
    _lib.call("kvbm_rope_kv_write", qkv.data_ptr(), T, hq, hkv, hd, positions.data_ptr(), cos_sin.data_ptr(),
              k_base or None, v_base or None, block_stride, token_stride, head_stride, page,
              slots.data_ptr() if slots is not None else None, _stream(stream))


def rope_kv_write_qout(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, hq: int, hkv: int,
                       k_base: int, v_base: int, block_stride: int, token_stride: int, head_stride: int, page: int,
                       slots: torch.Tensor, q_out: torch.Tensor, stream=None) -> torch.Tensor:
    """Decode form of the RoPE/KV kernel: K/V into the paged cache, rotated q into ``q_out`` [T, hq, 128]."""
    T = qkv.shape[0]
    if qkv.shape[-1] != 128 or q_out.shape != (T, hq, 128) or not q_out.is_contiguous():
        raise ValueError("rope_kv_write_qout needs head_dim 128 and a contiguous [T, hq, 128] q_out")
    _lib.call("kvbm_rope_kv_write_qout", qkv.data_ptr(), T, hq, hkv, positions.data_ptr(), cos_sin.data_ptr(),
              k_base or None, v_base or None, block_stride, token_stride, head_stride, page, slots.data_ptr(),
              q_out.data_ptr(), _stream(stream))
    return q_out


_SUBSETS = {"all": 0, "kv": 1, "q": 2}


def rope_kv_push(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, hq: int, hkv: int,
                 local: tuple | None, remote: tuple | None, r_head_offset: int = 0, heads: str = "all",
                 stream=None) -> None:
    """RoPE + KV write into ``local`` (optional) and ``remote`` (optional) paged caches in one kernel.

    Each cache is ``(k_base, v_base, block_stride, token_stride, head_stride,
    page, slots)`` with ``slots`` an int64 [T] tensor of block*page+offset
    (negative: skip). The remote cache may be a peer GPU's memory; its heads
    start at ``r_head_offset`` (a decode rank holding more KV heads than this
    prefill rank). ``heads`` restricts the launch to the K/V heads (``"kv"``:
    the part that moves KV) or the query heads (``"q"``). head_dim 128.
    """
    T = qkv.shape[0]
    if qkv.shape[-1] != 128:
        raise ValueError("rope_kv_push needs head_dim 128")
    lk = local or (0, 0, 0, 0, 0, 0, None)
    rk = remote or (0, 0, 0, 0, 0, 0, None)
    _lib.call("kvbm_rope_kv_push_heads", qkv.data_ptr(), T, hq, hkv, positions.data_ptr(), cos_sin.data_ptr(),
              lk[0] or None, lk[1] or None, lk[2], lk[3], lk[4], lk[5],
              lk[6].data_ptr() if lk[6] is not None else None,
              rk[0] or None, rk[1] or None, rk[2], rk[3], rk[4], rk[5], r_head_offset,
              rk[6].data_ptr() if rk[6] is not None else None, _SUBSETS[heads], _stream(stream))


def set_rope_unroll(unroll: int) -> int:
    """Head pairs per lane the RoPE/KV kernel keeps in flight (2, 4 or 8); returns the previous value."""
    prev = int(_lib.load().kvbm_rope_set_unroll(int(unroll)))
    if prev < 0:
        raise ValueError("unroll must be 2, 4 or 8")
    return prev


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    T = gate_up.numel() // gate_up.shape[-1]
    inter = gate_up.shape[-1] // 2
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], inter, dtype=gate_up.dtype, device=gate_up.device)
    _lib.call("kvbm_silu_mul", gate_up.data_ptr(), out.data_ptr(), T, inter, _stream(stream))
    return out


def decode_splits(batch: int, hkv: int, max_seq: int, page: int, sm_count: int = 148,
                  resident_per_sm: int = 2) -> int:
    """Number of KV splits for the decode attention grid (batch x hkv x splits CTAs).

    Starts from enough splits to fill the SMs about four times over, then
    looks at up to four times as many and keeps the one whose last wave of
    CTAs is fullest (``resident_per_sm`` CTAs of the tensor-core kernel fit
    on an SM), so the GPU does not idle on a ragged final wave.
    """
    blocks = max(1, (max_seq + page - 1) // page)
    groups = max(1, batch * hkv)
    slots = resident_per_sm * sm_count
    base = max(1, min(blocks, (4 * slots + groups - 1) // groups))
    best, best_eff = base, -1.0
    for s in range(base, min(blocks, 4 * base) + 1):
        waves = groups * s / slots
        eff = waves / math.ceil(waves)
        if eff > best_eff + 0.02:  # more splits cost partial writes: only for a clearly fuller last wave
            best, best_eff = s, eff
    return int(best)


def paged_decode_attn(q: torch.Tensor, k_base: int, v_base: int, block_stride: int, token_stride: int,
                      head_stride: int, page: int, block_table: torch.Tensor, seq_lens: torch.Tensor, hkv: int,
                      softmax_scale: float, splits: int, scratch: torch.Tensor | None = None,
                      out: torch.Tensor | None = None, stream=None, impl: str = "mma",
                      counters: torch.Tensor | None = None) -> torch.Tensor:
    """Split-KV paged decode attention. q: [B, Hq, 128] bf16; returns [B, Hq, 128].

    ``impl="mma"``: tensor-core kernel (mma.sync, cp.async-staged K/V);
    ``impl="simt"``: CUDA-core kernel (kept as the reference point).
    ``counters`` (int32, B * hkv zeros, reusable): the tensor-core kernel merges
    the splits in its last CTA per (request, KV head) instead of a second launch."""
    B, Hq, hd = q.shape
    if out is None:
        out = torch.empty_like(q)
    rows = B * Hq * splits
    need = rows * (hd + 2)
    if scratch is None or scratch.numel() < need:
        scratch = torch.empty(need, dtype=torch.float32, device=q.device)
    part_acc = scratch.data_ptr()
    part_ml = scratch.data_ptr() + rows * hd * 4
    args = (q.data_ptr(), k_base, v_base, block_stride, token_stride, head_stride, page, block_table.data_ptr(),
            block_table.shape[1], seq_lens.data_ptr(), B, Hq, hkv, hd, float(softmax_scale), splits, part_acc, part_ml)
    if impl == "mma" and counters is not None:
        if counters.dtype != torch.int32 or counters.numel() < B * hkv:
            raise ValueError("counters must be int32 with at least batch * hkv entries")
        _lib.call("kvbm_paged_decode_attn_fused", *args, counters.data_ptr(), out.data_ptr(), _stream(stream))
    else:
        _lib.call("kvbm_paged_decode_attn" if impl == "mma" else "kvbm_paged_decode_attn_simt", *args,
                  out.data_ptr(), _stream(stream))
    return out


class GemmWorkspace:
    """Scratch of :func:`skinny_gemm`: an fp32 [M, N] sum for tiles that several CTAs
    share and one ticket per 128-column tile, both zero between launches (the
    kernel re-zeroes what it used).

    One workspace serves launches that run one after another; GEMMs that may run
    at the same time (different streams) need one each."""

    def __init__(self, device, elems: int = 0, tiles: int = 0):
        self.device = torch.device(device)
        self.ws = torch.zeros(max(elems, 1), dtype=torch.float32, device=self.device)
        self.tickets = torch.zeros(max(tiles, 1), dtype=torch.int32, device=self.device)

    def reserve(self, elems: int, tiles: int) -> None:
        if self.ws.numel() < elems:
            self.ws = torch.zeros(elems, dtype=torch.float32, device=self.device)
        if self.tickets.numel() < tiles:
            self.tickets = torch.zeros(tiles, dtype=torch.int32, device=self.device)

    def clear(self) -> None:
        """Zero the partial sums and tickets (after a launch that gave up: an aborted CTA
        leaves its tile's ticket short and its partial sums in place)."""
        self.ws.zero_()
        self.tickets.zero_()


_workspaces: dict[int, GemmWorkspace] = {}


def skinny_gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, ctas: int = 0,
                workspace: GemmWorkspace | None = None, stream=None) -> torch.Tensor:
    """``out = x @ w.T`` for a few rows of x on the tcgen05 tensor cores (TMA-fed, TMEM accumulators).

    x: [M, K] bf16 with M <= 128 (a decode batch), w: [N, K] bf16; both with unit
    inner stride and 16-byte aligned rows. A persistent launch of ``ctas`` CTAs
    (0: one per SM) splits the weight's 128-row x 64-column chunks evenly among
    them (stream-K). Without ``workspace`` a per-device one is used, so
    concurrent launches on several streams must pass their own."""
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1]:
        raise ValueError(f"skinny_gemm shapes {tuple(x.shape)} x {tuple(w.shape)}^T")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("skinny_gemm takes bf16 operands")
    if x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("skinny_gemm operands need unit inner stride")
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    elif out.shape != (M, N) or out.stride(1) != 1 or out.dtype != torch.bfloat16:
        raise ValueError("skinny_gemm out must be bf16 [M, N] with unit inner stride")
    if workspace is None:
        dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
        workspace = _workspaces.get(dev)
        if workspace is None:
            workspace = _workspaces[dev] = GemmWorkspace(x.device)
    workspace.reserve(M * N, -(-N // 128))
    _lib.call("kvbm_skinny_gemm", x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
              out.stride(0), M, N, K, int(ctas), workspace.ws.data_ptr(), workspace.tickets.data_ptr(),
              _stream(stream))
    return out


def skinny_gemm_status(reset: bool = True) -> int:
    """0, or the error a :func:`skinny_gemm` launch recorded (3: a pipeline wait timed out). Synchronizes.

    A launch that gave up leaves its workspace dirty (partial sums, a ticket
    count that never reached the last CTA). With ``reset`` and a nonzero
    status, the per-device workspaces used when no ``workspace`` is passed are
    zeroed here; callers that pass their own workspace must call its
    :meth:`GemmWorkspace.clear` before the next launch."""
    st = int(_lib.load().kvbm_skinny_gemm_status(1 if reset else 0))
    if st and reset:
        for ws in _workspaces.values():
            ws.clear()
        torch.cuda.synchronize()
    return st


def set_skinny_gemm_pdl(on: bool) -> bool:
    """Launch :func:`skinny_gemm` with programmatic dependent launch (default on): its CTAs
    start streaming weights while the preceding kernel drains. Returns the previous setting."""
    return bool(_lib.load().kvbm_skinny_gemm_set_pdl(1 if on else 0))


_GEMM_MODES = {"auto": 0, "streamk": 1, "cluster": 2}


def set_skinny_gemm_mode(mode: str) -> str:
    """How :func:`skinny_gemm` splits the work: ``"auto"`` (estimated fastest, default),
    ``"streamk"`` (persistent CTAs, fp32 workspace fix-up) or ``"cluster"`` (thread-block
    clusters share a tile, partials summed through distributed shared memory).
    Returns the previous mode."""
    prev = int(_lib.load().kvbm_skinny_gemm_set_mode(_GEMM_MODES[mode]))
    return {v: k for k, v in _GEMM_MODES.items()}[prev]


_TIMELINE_SLOTS = ("entry", "prologue", "grid_dep", "first_stage", "last_mma", "last_drain", "fixup_done", "exit")


def skinny_gemm_timeline(run, device=None) -> dict:
    """Run ``run()`` (which should launch one stream-K :func:`skinny_gemm`) with per-CTA
    %globaltimer stamps on, and return per-phase statistics in microseconds since the
    earliest CTA entry: {phase: (median over CTAs, max over CTAs)}."""
    n_sm = torch.cuda.get_device_properties(device or torch.cuda.current_device()).multi_processor_count
    buf = torch.zeros(n_sm * 8, dtype=torch.int64, device=device or "cuda")
    lib = _lib.load()
    lib.kvbm_skinny_gemm_set_timeline(buf.data_ptr())
    try:
        run()
        torch.cuda.synchronize()
    finally:
        lib.kvbm_skinny_gemm_set_timeline(None)
    t = buf.view(n_sm, 8).cpu()
    used = t[:, 0] > 0
    t = t[used]
    t0 = int(t[:, 0].min())
    out = {}
    for i, name in enumerate(_TIMELINE_SLOTS):
        col = t[:, i]
        col = col[col > 0]
        if col.numel():
            rel = (col - t0).double() / 1e3
            out[name] = (round(float(rel.median()), 2), round(float(rel.max()), 2))
    out["ctas"] = int(used.sum())
    return out
