"""Tensor-level block permutes: the ``kvbm.kernels`` Python API over this library's sm_100a kernels.

A *block stack* is one block's KV as ``nl * no`` CUDA tensors (layer-major, K/V
minor), each a chunk shaped ``[nt, nh, hd]`` (``layout="NHD"``) or
``[nh, nt, hd]`` (``"HND"``). A *universal* block is one tensor
``[nh, nl, no, nt, hd]``; an *operational* block is one tensor ``[nl, no,
inner]`` holding the chunks back to back in their own layout.

* :func:`block_to_universal` / :func:`universal_to_block` - the permute
  kernels (one launch for all blocks, pointer tables on the device);
* :func:`block_to_operational` / :func:`operational_to_block` - chunk copies
  (``backend="kernel"``: the split-by-bytes pair-copy kernel on every SM;
  ``"async"``: one ``cudaMemcpyAsync`` per chunk on the copy engines;
  ``"auto"``/None: the kernel).

Every call runs on the current stream and synchronises it before returning,
as the reference's functions do, so the outputs are ready on return.

Parity: src/kernels.rs of the reference (block_to_universal,
universal_to_block, block_to_operational, operational_to_block and their
argument conventions: groups of chunk tensors, a single universal tensor
meaning one block, the layout strings and the backend names).
"""

from __future__ import annotations

from typing import Sequence

import torch

from .ops import kv_ops

_LAYOUT = {"NHD": 0, "HND": 1}


def _layout(layout: str) -> int:
    try:
        return _LAYOUT[layout.upper()]
    except (KeyError, AttributeError):
        raise ValueError(f"layout must be 'NHD' or 'HND', got {layout!r}") from None


def _groups(blocks) -> list[list[torch.Tensor]]:
    """``blocks`` as nb groups of chunk tensors (one group when a flat list of tensors is given)."""
    if isinstance(blocks, torch.Tensor):
        raise TypeError("blocks must be a sequence of per-block sequences of chunk tensors")
    groups = list(blocks)
    if groups and isinstance(groups[0], torch.Tensor):
        groups = [groups]
    return [list(g) for g in groups]


def _singles(ts) -> list[torch.Tensor]:
    return [ts] if isinstance(ts, torch.Tensor) else list(ts)


def _check_cuda(ts: Sequence[torch.Tensor], what: str) -> None:
    for t in ts:
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{what} must be contiguous CUDA tensors")


def _ptrs(ts: Sequence[torch.Tensor], device: torch.device) -> torch.Tensor:
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64).to(device)


def _chunk_geometry(chunk: torch.Tensor, layout: int) -> tuple[int, int, int]:
    """(nt, nh, hd) of one chunk tensor in ``layout``."""
    if chunk.dim() != 3:
        raise ValueError(f"chunk tensors are [nt, nh, hd] or [nh, nt, hd], got shape {tuple(chunk.shape)}")
    a, b, hd = chunk.shape
    return (a, b, hd) if layout == 0 else (b, a, hd)


def _permute(blocks, universals, layout: str, to_universal: bool) -> None:
    lay = _layout(layout)
    groups, unis = _groups(blocks), _singles(universals)
    if len(groups) != len(unis):
        raise ValueError(f"{len(groups)} block groups but {len(unis)} universal tensors")
    if not groups:
        return
    u0 = unis[0]
    if u0.dim() != 5:
        raise ValueError(f"universal tensors are [nh, nl, no, nt, hd], got shape {tuple(u0.shape)}")
    nh, nl, no, nt, hd = u0.shape
    chunks = [c for g in groups for c in g]
    _check_cuda(chunks, "block chunks")
    _check_cuda(unis, "universal tensors")
    if any(len(g) != nl * no for g in groups):
        raise ValueError(f"every block group needs nl * no = {nl * no} chunk tensors")
    if any(tuple(u.shape) != tuple(u0.shape) or u.dtype != u0.dtype for u in unis):
        raise ValueError("universal tensors differ in shape or dtype")
    for c in chunks:
        if _chunk_geometry(c, lay) != (nt, nh, hd) or c.dtype != u0.dtype:
            raise ValueError(f"chunk {tuple(c.shape)} {c.dtype} does not match the universal [nh={nh}, nt={nt}, "
                             f"hd={hd}] {u0.dtype} in layout {layout}")
    dev = u0.device
    with torch.cuda.device(dev):
        up, bp = _ptrs(unis, dev), _ptrs(chunks, dev)
        fn = kv_ops.universal_from_block if to_universal else kv_ops.block_from_universal
        fn(up, bp, nh, nl, no, nt, hd, u0.dtype, lay)
        torch.cuda.current_stream(dev).synchronize()


def block_to_universal(blocks, universals, layout: str = "NHD") -> None:
    """Gather each block's ``nl * no`` chunks into its universal ``[nh, nl, no, nt, hd]`` tensor."""
    _permute(blocks, universals, layout, True)


def universal_to_block(universals, blocks, layout: str = "NHD") -> None:
    """Scatter each universal ``[nh, nl, no, nt, hd]`` tensor into its block's chunks (inverse)."""
    _permute(blocks, universals, layout, False)


def _backend(backend: str | None) -> str:
    b = (backend or "auto").lower()
    if b not in ("auto", "kernel", "async", "batch"):
        raise ValueError(f"backend must be auto, kernel, async or batch, got {backend!r}")
    # one cudaMemcpyAsync per chunk stands in for a batched copy-engine call
    return "async" if b in ("async", "batch") else "kernel"


def _operational(blocks, operationals, backend: str | None, to_operational: bool) -> None:
    engine = _backend(backend)
    groups, ops = _groups(blocks), _singles(operationals)
    if len(groups) != len(ops):
        raise ValueError(f"{len(groups)} block groups but {len(ops)} operational tensors")
    if not groups:
        return
    chunks = [c for g in groups for c in g]
    _check_cuda(chunks, "block chunks")
    _check_cuda(ops, "operational tensors")
    csize = chunks[0].numel() * chunks[0].element_size()
    if any(c.numel() * c.element_size() != csize for c in chunks):
        raise ValueError("chunks differ in size")
    pairs_src, pairs_dst = [], []
    for g, op in zip(groups, ops):
        if op.numel() * op.element_size() != len(g) * csize:
            raise ValueError(f"operational tensor holds {op.numel() * op.element_size()} bytes, its block "
                             f"{len(g) * csize}")
        base = op.data_ptr()
        for i, c in enumerate(g):
            off = base + i * csize
            pairs_src.append(c.data_ptr() if to_operational else off)
            pairs_dst.append(off if to_operational else c.data_ptr())
    dev = ops[0].device
    with torch.cuda.device(dev):
        if engine == "kernel":
            kv_ops.copy_pairs(pairs_src, pairs_dst, csize)
        else:
            kv_ops.memcpy_pairs_ce(pairs_src, pairs_dst, csize)
        torch.cuda.current_stream(dev).synchronize()


def block_to_operational(blocks, operationals, backend: str | None = None) -> None:
    """Copy each block's chunks back to back into its operational ``[nl, no, inner]`` tensor."""
    _operational(blocks, operationals, backend, True)


def operational_to_block(operationals, blocks, backend: str | None = None) -> None:
    """Copy each operational tensor's chunks back into the block's chunk tensors (inverse)."""
    _operational(blocks, operationals, backend, False)


__all__ = ["block_to_universal", "universal_to_block", "block_to_operational", "operational_to_block"]
