"""Transfer planning: what a block transfer between two layouts needs, and
which engine runs it.

* :func:`plan_copy` classifies a transfer; when no transform is needed its
  ``ops()`` are byte-range copies: one per block when both pools hold whole
  blocks contiguously, else one per (block, layer, outer) chunk, with adjacent
  ranges that are contiguous on both sides merged.
  ``TRANSFORM`` plans (layout permutes, KV-head slices, dtype casts) have no
  byte ranges: a kernel computes every address.
* :func:`lower` picks the engine: the copy engines when asked to, the
  split-by-bytes pair-copy kernel for same-layout whole blocks, the tile kernel
  for dtype casts (issue-bound fp8 work), the TMA-staged pipeline otherwise;
  a startup-benchmark result overrides the default where one exists. It also
  reports whether the plan's runs are large enough for DMA
  (``CopyPolicy.min_inner_bytes``).
* :class:`PreparedPlanCache` memoises engine choices per (layout pair, layer
  range, head range), LRU-bounded.

Parity: crates/kvbm-physical/src/transfer/plan.rs (CopyOp, CopyPlan
{Direct, Transform, Staged}, CopyPolicy{min_inner_bytes = 4 KiB, coalesce}; Staged plans
are the two-hop strategies of physical/transfer.py),
plan_copy), transfer/lower.rs (candidates and their selection),
transfer/prepared.rs (PreparedPlanCache).
"""

from __future__ import annotations

import enum
from collections import OrderedDict
from dataclasses import dataclass

from .layout import KvBlockLayout, KvLayout


@dataclass(frozen=True)
class CopyOp:
    src: int
    dst: int
    size: int


@dataclass
class CopyPolicy:
    min_inner_bytes: int = 4096  # smaller contiguous runs go to an SM kernel, not a DMA engine


class PlanKind(str, enum.Enum):
    DIRECT = "direct"        # byte-range copies, no data changes
    TRANSFORM = "transform"  # a kernel rewrites addresses (permute, head slice) or values (fp8)


@dataclass
class CopyPlan:
    kind: PlanKind
    reason: str
    bytes: int
    whole_blocks: bool = False  # DIRECT: one range per block (else one per (block, layer, outer) chunk)
    unit: int = 0               # DIRECT: bytes per range before coalescing
    _args: tuple | None = None  # (src, src_ids, dst, dst_ids, layer begin, layer end), for ops()

    def ops(self, coalesced: bool = True) -> list[CopyOp]:
        """The byte ranges of a DIRECT plan (built on demand: one per block or chunk)."""
        if self.kind != PlanKind.DIRECT or self._args is None:
            return []
        src, src_ids, dst, dst_ids, lb, le = self._args
        if self.whole_blocks:
            out = [CopyOp(src.layer_base(0) + s * src.block_stride, dst.layer_base(0) + d * dst.block_stride,
                          self.unit) for s, d in zip(src_ids, dst_ids)]
        else:
            out = []
            for s, d in zip(src_ids, dst_ids):
                for l in range(lb, le):
                    for o in range(src.config.outer_dim):
                        sa, size = src.memory_region(s, l, o)
                        out.append(CopyOp(sa, dst.memory_region(d, l, o)[0], size))
        return coalesce(out) if coalesced else out


def coalesce(ops: list[CopyOp]) -> list[CopyOp]:
    """Merge consecutive ops whose source and destination ranges both continue the previous op."""
    out: list[CopyOp] = []
    for o in ops:
        if out and out[-1].src + out[-1].size == o.src and out[-1].dst + out[-1].size == o.dst:
            p = out[-1]
            out[-1] = CopyOp(p.src, p.dst, p.size + o.size)
        else:
            out.append(o)
    return out


def same_geometry(a: KvLayout, b: KvLayout) -> bool:
    ca, cb = a.config, b.config
    return (ca.num_layers, ca.outer_dim, ca.page_size, ca.inner_dim, ca.dtype_width_bytes) == (
        cb.num_layers, cb.outer_dim, cb.page_size, cb.inner_dim, cb.dtype_width_bytes)


def plan_copy(src: KvLayout, src_ids, dst: KvLayout, dst_ids, layer_range: tuple[int, int] | None = None,
              head_range: tuple[int, int, int] | None = None) -> CopyPlan:
    """Classify a transfer (O(1)); the byte ranges of a DIRECT plan come from ``plan.ops()``."""
    if len(src_ids) != len(dst_ids):
        raise ValueError("source and destination id lists differ in length")
    lb, le = layer_range or (0, src.config.num_layers)
    nbytes = len(src_ids) * (le - lb) * src.config.outer_dim * src.config.bytes_per_chunk
    whole = (src.kind == dst.kind == "fully_contiguous" and (lb, le) == (0, src.config.num_layers)
             and src.block_stride == src.config.bytes_per_block and dst.block_stride == dst.config.bytes_per_block)
    why = None
    if src.dtype != dst.dtype:
        why = "dtype cast"
    elif src.block_layout != dst.block_layout:
        why = "block layout permute"
    elif head_range is not None:
        why = "KV-head slice"
    elif not same_geometry(src, dst):
        why = "geometry differs"
    elif src.block_layout == KvBlockLayout.UNIVERSAL and not whole:
        why = "universal blocks have no contiguous (layer, outer) chunks"
    if why is not None:
        return CopyPlan(PlanKind.TRANSFORM, why, nbytes)
    # whole blocks: the bytes move unchanged whatever the block layout
    unit = src.config.bytes_per_block if whole else src.config.bytes_per_chunk
    return CopyPlan(PlanKind.DIRECT, "same layout", nbytes, whole, unit, (src, src_ids, dst, dst_ids, lb, le))


@dataclass
class Lowered:
    engine: str           # ce | pairs | tile | tma
    dma_ok: bool          # runs are at least CopyPolicy.min_inner_bytes (copy engines are efficient)
    plan: CopyPlan


def lower(plan: CopyPlan, src: KvLayout, dst: KvLayout, *, prefer_copy_engine: bool = False, engine: str = "auto",
          bench_choice: str | None = None, policy: CopyPolicy | None = None) -> Lowered:
    """The engine for a plan. ``engine`` != "auto" forces one; ``bench_choice`` is a
    startup-benchmark result for this layout pair (or None)."""
    policy = policy or CopyPolicy()
    dma_ok = plan.kind == PlanKind.DIRECT and plan.unit >= policy.min_inner_bytes  # coalescing only grows runs
    if engine != "auto":
        return Lowered(engine, dma_ok, plan)
    if prefer_copy_engine:
        return Lowered("ce", dma_ok, plan)
    if plan.kind == PlanKind.DIRECT and plan.whole_blocks:
        return Lowered("pairs", dma_ok, plan)
    if bench_choice is not None:
        return Lowered(bench_choice, dma_ok, plan)
    if src.dtype != dst.dtype:
        # fp8 casts are issue-bound, not copy-bound: the tile kernel's 8 resident CTAs per SM
        # beat the TMA pipe's one producer + 8 consumer warps (3.8 vs 3.1 TB/s quantising,
        # 4.2 vs 3.3 TB/s dequantising, 128 Llama-3-8B blocks on B200)
        return Lowered("tile", dma_ok, plan)
    return Lowered("tma", dma_ok, plan)


def layout_signature(lay: KvLayout) -> tuple:
    """What an engine choice depends on: geometry, block layout, dtype, strides, placement."""
    c = lay.config
    return (lay.kind, lay.block_layout, lay.dtype, lay.block_stride, lay.base_ptr, lay.location, c.num_layers,
            c.outer_dim, c.page_size, c.inner_dim, c.dtype_width_bytes, c.num_blocks)


class PreparedPlanCache:
    """LRU of engine choices keyed by (layout signatures, layer range, head range, forced
    engine): a choice does not depend on the block ids, so repeated transfers between the
    same pools skip planning."""

    def __init__(self, capacity: int = 256):
        self.capacity = capacity
        self._d: OrderedDict[tuple, Lowered] = OrderedDict()
        self.hits = self.misses = 0

    @staticmethod
    def key(src: KvLayout, dst: KvLayout, layer_range, head_range, engine: str) -> tuple:
        lr = tuple(layer_range) if layer_range is not None else None  # callers may pass lists
        hr = tuple(head_range) if head_range is not None else None
        return (layout_signature(src), layout_signature(dst), lr, hr, engine)

    def get(self, key: tuple) -> Lowered | None:
        v = self._d.get(key)
        if v is None:
            self.misses += 1
            return None
        self._d.move_to_end(key)
        self.hits += 1
        return v

    def put(self, key: tuple, value: Lowered) -> None:
        self._d[key] = value
        self._d.move_to_end(key)
        while len(self._d) > self.capacity:
            self._d.popitem(last=False)

    def clear(self) -> None:
        self._d.clear()
