"""Llama-architecture driver harness (random-init weights) whose KV cache
lives in a block manager pool.

The model exists to exercise the block manager the way a serving engine
does: prefill writes K/V into paged blocks layer by layer (and lets a
callback start the transfer of each finished layer), decode attends over
paged blocks through a block table. GEMMs go to cuBLAS (``F.linear``),
prefill attention to PyTorch SDPA (flash / cuDNN backends only), and the
fused ops (RMSNorm+residual, RoPE+paged KV write, SiLU-mul, paged decode
attention) to the sm_100a kernels in ``libkvbm_cuda.so``.

The reference ships no model (vLLM provides it there); this harness plays
vLLM's role for the benchmarks, calling the same connector hooks.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel
from torch.nn.attention.bias import causal_lower_right

from ..ops import llama_ops
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig


@dataclass(frozen=True)
class LlamaConfig:
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5
    max_position: int = 16384

    @classmethod
    def llama3_8b(cls) -> "LlamaConfig":
        return cls()

    @classmethod
    def tiny(cls, layers: int = 2) -> "LlamaConfig":
        return cls(hidden=512, layers=layers, heads=8, kv_heads=2, head_dim=128, intermediate=1024, vocab=1024,
                   max_position=4096)

    @property
    def q_size(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    def kv_layout_config(self, num_blocks: int, page_size: int = 16,
                         dtype: torch.dtype = torch.bfloat16) -> LayoutConfig:
        return LayoutConfig.for_model(num_blocks, self.layers, self.kv_heads, self.head_dim, page_size, dtype)

    def num_params(self) -> int:
        per_layer = (self.hidden * (self.q_size + 2 * self.kv_size) + self.q_size * self.hidden
                     + 3 * self.hidden * self.intermediate + 2 * self.hidden)
        return self.layers * per_layer + 2 * self.vocab * self.hidden + self.hidden


class KvPush:
    """Destination of the K/V a prefill produces, written by the RoPE/KV kernel itself.

    ``remote`` is the decode instance's pool (mapped through CUDA IPC when it
    is on another GPU); ``block_ids`` (int32, device) are its blocks for the
    request, one per ``page`` tokens. Each layer is two launches of the
    RoPE/KV kernel: the K/V heads (rotated K and V stored into ``remote``,
    K rotated in place for the attention) and then the query heads. With
    ``timers`` set, the K/V launch is bracketed by CUDA events and
    ``(start, end, kv_bytes)`` appended, so callers can report the device
    time of the transfer.
    """

    def __init__(self, remote: KvLayout, block_ids: torch.Tensor, *, start_pos: int = 0, head_offset: int = 0,
                 local_write: bool = False, timers: list | None = None):
        if remote.dtype != torch.bfloat16:
            raise ValueError("the fused push writes bf16 pools; use the transfer kernels for fp8")
        self.remote, self.block_ids = remote, block_ids
        self.start_pos, self.head_offset = start_pos, head_offset
        self.local_write, self.timers = local_write, timers
        self._slots: torch.Tensor | None = None

    def slots(self, pos: torch.Tensor) -> torch.Tensor:
        if self._slots is None or self._slots.numel() != pos.numel():
            page = self.remote.config.page_size
            p = pos.long()
            self._slots = self.block_ids.long()[p // page] * page + p % page
        return self._slots

    def layer(self, model: "LlamaModel", li: int, qkv: torch.Tensor, pos: torch.Tensor, local: tuple) -> None:
        c = model.cfg
        r = self.remote
        rk = r.layer_base(li)
        remote = (rk, rk + r.outer_stride, r.block_stride, r.token_stride, r.head_stride, r.config.page_size,
                  self.slots(pos))
        ev = None
        split = c.heads % 2 == 0  # K/V heads in their own launch, query heads after it
        if self.timers is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        llama_ops.rope_kv_push(qkv, pos, model.cos_sin, c.heads, c.kv_heads, local if self.local_write else None,
                               remote, r_head_offset=self.head_offset, heads="kv" if split else "all")
        if ev is not None:
            ev[1].record()
            self.timers.append((ev[0], ev[1], qkv.shape[0] * 2 * c.kv_heads * c.head_dim * 2))
        if split:
            llama_ops.rope_kv_push(qkv, pos, model.cos_sin, c.heads, c.kv_heads, None, None, heads="q")


class LlamaModel:
    """Weights + forward passes. Not an nn.Module: no autograd, inference only.

    With ``tp_size`` > 1 the model is this rank's tensor-parallel shard:
    ``heads / tp`` query heads and ``kv_heads / tp`` KV heads (the rank's KV
    pool holds only those), ``intermediate / tp`` FFN columns; the attention
    output and FFN down projections are row-parallel and summed over
    ``tp_group`` with an all-reduce (NCCL). ``self.cfg`` is the shard's
    geometry, ``self.full_cfg`` the model's. ``shard_init="slice"`` draws
    every weight at full size from ``seed`` and keeps this rank's slice, so
    any TP degree computes the same model as TP = 1 (up to the order of the
    all-reduce sums); ``"independent"`` draws only the shard (models too
    large to materialise whole on one GPU).
    """

    def __init__(self, cfg: LlamaConfig, device: torch.device | str = "cuda", seed: int = 0,
                 dtype: torch.dtype = torch.bfloat16, tp_rank: int = 0, tp_size: int = 1, tp_group=None,
                 shard_init: str = "slice"):
        if cfg.heads % tp_size or cfg.kv_heads % tp_size or cfg.intermediate % tp_size:
            raise ValueError(f"tp_size {tp_size} must divide heads, kv_heads and intermediate")
        self.full_cfg = cfg
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        if tp_size > 1:
            from dataclasses import replace

            cfg = replace(cfg, heads=cfg.heads // tp_size, kv_heads=cfg.kv_heads // tp_size,
                          intermediate=cfg.intermediate // tp_size)
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        sliced = tp_size == 1 or shard_init == "slice"
        g = torch.Generator(device=self.device).manual_seed(seed if sliced else seed + 7919 * tp_rank)
        std = 0.02

        def w(*shape, scale=std):
            t = torch.empty(shape, device=self.device, dtype=dtype)
            t.normal_(0.0, scale, generator=g)
            return t

        c, F_ = cfg, self.full_cfg
        T, r = tp_size, tp_rank

        def rows(t, parts):
            """This rank's slice of each of ``parts`` consecutive row blocks of t."""
            out, o = [], 0
            for n in parts:
                k = n // T
                out.append(t[o + r * k: o + (r + 1) * k])
                o += n
            return torch.cat(out).contiguous()

        def layer_weights():
            if sliced:
                wqkv = w(F_.q_size + 2 * F_.kv_size, F_.hidden)
                wo = w(F_.hidden, F_.q_size, scale=std / math.sqrt(2 * F_.layers))
                wgu = w(2 * F_.intermediate, F_.hidden)
                wd = w(F_.hidden, F_.intermediate, scale=std / math.sqrt(2 * F_.layers))
                if T > 1:
                    wqkv = rows(wqkv, [F_.q_size, F_.kv_size, F_.kv_size])
                    wo = wo[:, r * c.q_size:(r + 1) * c.q_size].contiguous()
                    wgu = rows(wgu, [F_.intermediate, F_.intermediate])
                    wd = wd[:, r * c.intermediate:(r + 1) * c.intermediate].contiguous()
                return wqkv, wo, wgu, wd
            return (w(c.q_size + 2 * c.kv_size, c.hidden), w(c.hidden, c.q_size, scale=std / math.sqrt(2 * c.layers)),
                    w(2 * c.intermediate, c.hidden), w(c.hidden, c.intermediate, scale=std / math.sqrt(2 * c.layers)))

        g_rep = torch.Generator(device=self.device).manual_seed(seed)  # replicated tensors: same on every rank
        self.embed = torch.empty(c.vocab, c.hidden, device=self.device, dtype=dtype).normal_(0.0, std, generator=g_rep)
        self.layers = []
        for _ in range(c.layers):
            wqkv, wo, wgu, wd = layer_weights()
            self.layers.append({
                "wqkv": wqkv, "wo": wo, "wgu": wgu, "wd": wd,
                "n1": torch.ones(c.hidden, device=self.device, dtype=dtype),
                "n2": torch.ones(c.hidden, device=self.device, dtype=dtype),
            })
        self.norm = torch.ones(c.hidden, device=self.device, dtype=dtype)
        self.lm_head = torch.empty(c.vocab, c.hidden, device=self.device, dtype=dtype).normal_(0.0, std,
                                                                                            generator=g_rep)
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.float64) / c.head_dim))
        f = torch.outer(torch.arange(c.max_position, dtype=torch.float64), inv)
        self.cos_sin = torch.cat([f.cos(), f.sin()], dim=-1).float().to(self.device)
        self.scale = 1.0 / math.sqrt(c.head_dim)
        self._decode_scratch: torch.Tensor | None = None
        self._decode_counters: torch.Tensor | None = None
        self.decode_gemm = "cublas"  # "tc": decode projections on the tcgen05 skinny GEMM
        self._gemm_ws: llama_ops.GemmWorkspace | None = None
        self._attn_backends: dict[bool, list] = {}

    # ------------------------------------------------------------ helpers
    def _reduce(self, x: torch.Tensor) -> torch.Tensor:
        """Sum a row-parallel projection's partial output over the tensor-parallel ranks."""
        if self.tp_size > 1:
            import torch.distributed as dist

            dist.all_reduce(x, group=self.tp_group)
        return x

    @staticmethod
    def kv_bases(pool: KvLayout, layer: int) -> tuple[int, int]:
        k = pool.layer_base(layer)
        return k, k + pool.outer_stride

    def allocate_pool(self, num_blocks: int, page_size: int = 16, kind: str = "fully_contiguous",
                      block_layout: KvBlockLayout = KvBlockLayout.OPERATIONAL_NHD) -> KvLayout:
        return KvLayout.allocate(self.cfg.kv_layout_config(num_blocks, page_size), kind, block_layout,
                                 device=self.device.index)

    # ------------------------------------------------------------ prefill
    @torch.inference_mode()
    def prefill(self, tokens: torch.Tensor, pool: KvLayout, block_ids: torch.Tensor, start_pos: int = 0,
                on_layer_done=None, kv_push: "KvPush | None" = None, on_layer_start=None) -> torch.Tensor:
        """Prefill ``tokens`` [T] at positions [start_pos, start_pos+T).

        K/V land in ``pool`` blocks ``block_ids`` (int32, device; block j holds
        positions [16j, 16j+16) of the sequence). ``on_layer_done(layer)`` is
        called on the host right after layer ``layer``'s K/V writes are enqueued
        on the current stream, ``on_layer_start(layer)`` before the layer reads
        the pool (a layer-wise onboard makes the stream wait for that layer
        there). With ``kv_push`` the kernel that rotates and
        writes each layer's K/V also stores it into ``kv_push.remote`` (a
        decode pool, possibly a peer GPU's), and the local pool write is
        skipped unless ``kv_push.local_write``. Returns the greedy next token
        (int64 [1]).
        """
        c = self.cfg
        T = tokens.numel()
        page = pool.config.page_size
        pos = torch.arange(start_pos, start_pos + T, device=self.device, dtype=torch.int32)
        slots = (block_ids.long()[pos.long() // page] * page + pos.long() % page)
        x = F.embedding(tokens.long(), self.embed)
        residual = x
        h = torch.empty_like(x)
        first = True
        for li, L in enumerate(self.layers):
            if on_layer_start is not None:
                on_layer_start(li)
            if first:
                llama_ops.rmsnorm(x, L["n1"], c.eps, out=h)
                first = False
            else:
                llama_ops.rmsnorm(x, L["n1"], c.eps, residual=residual, out=h)
            qkv = F.linear(h, L["wqkv"]).view(T, c.heads + 2 * c.kv_heads, c.head_dim)
            kb, vb = self.kv_bases(pool, li)
            if kv_push is None:
                llama_ops.rope_kv_write(qkv, pos, self.cos_sin, c.heads, c.kv_heads, c.head_dim, kb, vb,
                                        pool.block_stride, pool.token_stride, pool.head_stride, page, slots)
            else:
                kv_push.layer(self, li, qkv, pos, (kb, vb, pool.block_stride, pool.token_stride, pool.head_stride,
                                                   page, slots))
            if on_layer_done is not None:
                on_layer_done(li)
            q = qkv[:, : c.heads].transpose(0, 1).unsqueeze(0)
            k = qkv[:, c.heads: c.heads + c.kv_heads].transpose(0, 1)
            v = qkv[:, c.heads + c.kv_heads:].transpose(0, 1)
            if start_pos > 0:
                # cached prefix (e.g. onboarded from G2): read its K/V from the pool
                nb = (start_pos + page - 1) // page
                view = pool.layer_view(li)[block_ids[:nb].long()]  # [nb, 2, page, Hkv, D]
                pk = view[:, 0].reshape(-1, c.kv_heads, c.head_dim)[:start_pos].transpose(0, 1)
                pv = view[:, 1].reshape(-1, c.kv_heads, c.head_dim)[:start_pos].transpose(0, 1)
                k = torch.cat([pk, k], dim=1)
                v = torch.cat([pv, v], dim=1)
            a = self._attention(q, k.unsqueeze(0), v.unsqueeze(0), start_pos)
            a = a.squeeze(0).transpose(0, 1).reshape(T, c.q_size)
            x = self._reduce(F.linear(a, L["wo"]))
            llama_ops.rmsnorm(x, L["n2"], c.eps, residual=residual, out=h)
            gu = F.linear(h, L["wgu"])
            x = self._reduce(F.linear(llama_ops.silu_mul(gu), L["wd"]))
        last = torch.empty(1, c.hidden, device=self.device, dtype=self.dtype)
        res_last = residual[-1:].contiguous()
        llama_ops.rmsnorm(x[-1:].contiguous(), self.norm, c.eps, residual=res_last, out=last)
        logits = F.linear(last, self.lm_head)
        return logits.argmax(dim=-1)

    @property
    def attention_backend(self) -> str:
        """Backend the no-prefix prefill attention resolved to (after the first prefill)."""
        order = self._attn_backends.get(False, [SDPBackend.CUDNN_ATTENTION])
        return "expanded-heads" if not order or order[0] is None else order[0].name.lower()

    def _attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, offset: int) -> torch.Tensor:
        """Causal prefill attention, q [1, Hq, T, D] against k/v [1, Hkv, offset + T, D].

        cuDNN's fused attention with grouped-query heads runs this shape at
        about four times the rate of the flash backend on sm_100 (0.39 ms vs
        1.59 ms for 8,192 tokens, 32/8 heads). Backends that cannot take the
        shape (strides, GQA, the lower-right causal mask of a prefix) are
        skipped once and the next one is used from then on.
        """
        T, S = q.shape[2], k.shape[2]
        mask = None if offset == 0 else causal_lower_right(T, S)
        key = offset > 0
        order = self._attn_backends.get(key, [SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, None])
        for i, be in enumerate(order):
            try:
                if be is None:  # last resort: explicit head expansion for backends without GQA
                    rep = q.shape[1] // k.shape[1]
                    kk, vv = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
                    with sdpa_kernel([SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION,
                                      SDPBackend.MATH]):
                        if mask is None:
                            return F.scaled_dot_product_attention(q, kk, vv, is_causal=True, scale=self.scale)
                        return F.scaled_dot_product_attention(q, kk, vv, attn_mask=mask, scale=self.scale)
                with sdpa_kernel([be]):
                    if mask is None:
                        return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=self.scale,
                                                              enable_gqa=True)
                    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=self.scale, enable_gqa=True)
            except RuntimeError:
                self._attn_backends[key] = order[i + 1:]
        raise RuntimeError("no attention backend accepted the prefill shape")

    # ------------------------------------------------------------- decode
    def decode_scratch(self, batch: int, splits: int) -> torch.Tensor:
        need = batch * self.cfg.heads * splits * (self.cfg.head_dim + 2)
        if self._decode_scratch is None or self._decode_scratch.numel() < need:
            self._decode_scratch = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._decode_scratch

    def dlinear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """A decode-step projection ``x @ w.T``: the tcgen05 skinny GEMM for up to 128 rows
        (``decode_gemm == "tc"``), cuBLAS otherwise."""
        if self.decode_gemm == "tc" and x.shape[0] <= 128:
            if self._gemm_ws is None:
                self._gemm_ws = llama_ops.GemmWorkspace(self.device)
            return llama_ops.skinny_gemm(x, w, workspace=self._gemm_ws)
        return F.linear(x, w)

    def decode_counters(self, batch: int) -> torch.Tensor:
        """Zeroed split-merge tickets for the attention kernel (it leaves them zero after every launch)."""
        need = batch * self.cfg.kv_heads
        if self._decode_counters is None or self._decode_counters.numel() < need:
            self._decode_counters = torch.zeros(need, dtype=torch.int32, device=self.device)
        return self._decode_counters

    @torch.inference_mode()
    def decode_step(self, tokens: torch.Tensor, positions: torch.Tensor, pool: KvLayout, block_table: torch.Tensor,
                    seq_lens: torch.Tensor, splits: int) -> torch.Tensor:
        """One decode step for a batch: tokens [B] int64, positions [B] int32
        (position of each input token), block_table [B, max_blocks] int32,
        seq_lens [B] int32 (= positions + 1). Returns next tokens [B] int64.
        All shapes static, so the step can be captured in a CUDA graph."""
        c = self.cfg
        B = tokens.numel()
        page = pool.config.page_size
        pl = positions.long()
        slots = block_table.gather(1, (pl // page).unsqueeze(1)).squeeze(1).long() * page + pl % page
        x = F.embedding(tokens, self.embed)
        residual = x
        h = torch.empty_like(x)
        scratch = self.decode_scratch(B, splits)
        counters = self.decode_counters(B)
        attn = torch.empty(B, c.heads, c.head_dim, device=self.device, dtype=self.dtype)
        q = torch.empty(B, c.heads, c.head_dim, device=self.device, dtype=self.dtype)
        for li, L in enumerate(self.layers):
            if li == 0:
                llama_ops.rmsnorm(x, L["n1"], c.eps, out=h)
            else:
                llama_ops.rmsnorm(x, L["n1"], c.eps, residual=residual, out=h)
            qkv = self.dlinear(h, L["wqkv"]).view(B, c.heads + 2 * c.kv_heads, c.head_dim)
            kb, vb = self.kv_bases(pool, li)
            if c.head_dim == 128:
                llama_ops.rope_kv_write_qout(qkv, positions, self.cos_sin, c.heads, c.kv_heads, kb, vb,
                                             pool.block_stride, pool.token_stride, pool.head_stride, page, slots, q)
            else:
                llama_ops.rope_kv_write(qkv, positions, self.cos_sin, c.heads, c.kv_heads, c.head_dim, kb, vb,
                                        pool.block_stride, pool.token_stride, pool.head_stride, page, slots)
                q.copy_(qkv[:, : c.heads])
            llama_ops.paged_decode_attn(q, kb, vb, pool.block_stride, pool.token_stride, pool.head_stride, page,
                                        block_table, seq_lens, c.kv_heads, self.scale, splits, scratch=scratch,
                                        out=attn, counters=counters)
            x = self._reduce(self.dlinear(attn.view(B, c.q_size), L["wo"]))
            llama_ops.rmsnorm(x, L["n2"], c.eps, residual=residual, out=h)
            x = self._reduce(self.dlinear(llama_ops.silu_mul(self.dlinear(h, L["wgu"])), L["wd"]))
        out = torch.empty_like(h)
        llama_ops.rmsnorm(x, self.norm, c.eps, residual=residual, out=out)
        return self.dlinear(out, self.lm_head).argmax(dim=-1)

    # ---------------------------------------------------- torch reference
    @torch.inference_mode()
    def reference_forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Plain PyTorch (fp32 accumulate) causal forward; logits of every position."""
        c = self.cfg
        T = tokens.numel()
        x = F.embedding(tokens.long(), self.embed).float()
        pos = torch.arange(T, device=self.device)
        cs = self.cos_sin[pos]
        cos, sin = cs[:, None, : c.head_dim // 2], cs[:, None, c.head_dim // 2:]

        def rope(t):
            t1, t2 = t[..., : c.head_dim // 2], t[..., c.head_dim // 2:]
            return torch.cat([t1 * cos - t2 * sin, t2 * cos + t1 * sin], dim=-1)

        def norm(t, wgt):
            return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + c.eps) * wgt.float()

        for L in self.layers:
            hN = norm(x, L["n1"])
            qkv = (hN @ L["wqkv"].float().t()).view(T, -1, c.head_dim)
            q = rope(qkv[:, : c.heads])
            k = rope(qkv[:, c.heads: c.heads + c.kv_heads])
            v = qkv[:, c.heads + c.kv_heads:]
            rep = c.heads // c.kv_heads
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
            s = torch.einsum("thd,shd->hts", q, k) * self.scale
            mask = torch.triu(torch.ones(T, T, device=self.device, dtype=torch.bool), 1)
            s = s.masked_fill(mask, float("-inf"))
            a = torch.einsum("hts,shd->thd", s.softmax(-1), v).reshape(T, c.q_size)
            x = x + a @ L["wo"].float().t()
            hN = norm(x, L["n2"])
            gu = hN @ L["wgu"].float().t()
            x = x + (F.silu(gu[:, : c.intermediate]) * gu[:, c.intermediate:]) @ L["wd"].float().t()
        return norm(x, self.norm) @ self.lm_head.float().t()
