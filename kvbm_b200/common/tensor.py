"""Labelled KV tensor algebra shared by the connector, the layouts and the
transfer planner.

* :class:`KvDim` names the axes a KV cache tensor can have.
* :class:`KvDimLayout` is a labelled, sized axis list with its invariants
  checked once (one block axis, outer of size 1 or 2, payload last, ...).
* :class:`KvDimStrides` holds the byte strides of such a tensor and answers
  the question the copy planner asks: how many trailing bytes are one
  contiguous run (the unit a copy can move without a gather).
* :class:`AxisSlice` / :func:`intersect_axis` describe a rank's window of a
  sharded axis (KV heads under tensor parallelism) in global coordinates and
  the overlap of two windows in each side's local coordinates: the head
  ranges a heterogeneous-TP transfer must move between two ranks.
* :class:`LayoutSignature` summarises a layout for compatibility checks.
* :class:`CoordByLabel`, :class:`CanonicalBlockShape`,
  :class:`LogicalLayoutHandle` and :class:`KvbmTransferRoute` are the small
  value types the rest of the engine exchanges.

Parity: crates/kvbm-common/src/{tensor.rs (KvDim, KvDimLayout),
strides.rs (KvDimStrides), slice.rs (AxisSlice, AxisExtent,
AxisIntersection, intersect_axis, LayoutSignature), coord.rs, shape.rs,
lib.rs (LogicalLayoutHandle, KvbmTransferRoute)}.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import Sequence


class KvDim(str, enum.Enum):
    BLOCK = "block"
    LAYER = "layer"
    OUTER = "outer"
    PAGE = "page"
    HEAD = "head_count"
    HEAD_SIZE = "head_size"
    PAYLOAD = "payload"  # opaque trailing bytes (packed / quantised formats)


class LogicalLayoutHandle(enum.Enum):
    G1 = "g1"  # device memory
    G2 = "g2"  # pinned host memory
    G3 = "g3"  # local disk
    G4 = "g4"  # external object store


class KvbmTransferRoute(enum.Enum):
    """Metric labels of tier moves: offload goes down the tiers, onboard up."""

    OFFLOAD_D2H = "offload_d2h"   # G1 -> G2
    OFFLOAD_H2D = "offload_h2d"   # G2 -> G3 (host to disk)
    OFFLOAD_D2D = "offload_d2d"   # G1 -> G3
    OFFLOAD_D2O = "offload_d2o"   # -> G4
    ONBOARD_D2H = "onboard_d2h"   # G3 -> G2 (disk to host)
    ONBOARD_H2D = "onboard_h2d"   # G2 -> G1
    ONBOARD_D2D = "onboard_d2d"   # G3 -> G1
    ONBOARD_O2D = "onboard_o2d"   # G4 ->

    @classmethod
    def of(cls, src: LogicalLayoutHandle, dst: LogicalLayoutHandle) -> "KvbmTransferRoute":
        G = LogicalLayoutHandle
        table = {(G.G1, G.G2): cls.OFFLOAD_D2H, (G.G2, G.G3): cls.OFFLOAD_H2D, (G.G1, G.G3): cls.OFFLOAD_D2D,
                 (G.G2, G.G4): cls.OFFLOAD_D2O, (G.G1, G.G4): cls.OFFLOAD_D2O, (G.G3, G.G4): cls.OFFLOAD_D2O,
                 (G.G3, G.G2): cls.ONBOARD_D2H, (G.G2, G.G1): cls.ONBOARD_H2D, (G.G3, G.G1): cls.ONBOARD_D2D,
                 (G.G4, G.G1): cls.ONBOARD_O2D, (G.G4, G.G2): cls.ONBOARD_O2D, (G.G4, G.G3): cls.ONBOARD_O2D}
        try:
            return table[(src, dst)]
        except KeyError:
            raise ValueError(f"no route {src.name} -> {dst.name}") from None


@dataclass(frozen=True)
class KvDimLayout:
    dims: tuple[KvDim, ...]
    sizes: tuple[int, ...]

    def __init__(self, dims: Sequence[KvDim], sizes: Sequence[int]):
        dims, sizes = tuple(KvDim(d) for d in dims), tuple(int(s) for s in sizes)
        if not dims or len(dims) != len(sizes):
            raise ValueError(f"dims {dims} and sizes {sizes} must be non-empty and of equal length")
        if any(s <= 0 for s in sizes):
            raise ValueError(f"every size must be positive: {sizes}")
        counts = {d: dims.count(d) for d in KvDim}
        if counts[KvDim.BLOCK] != 1:
            raise ValueError("exactly one block axis required")
        for d in (KvDim.LAYER, KvDim.OUTER, KvDim.PAGE, KvDim.HEAD):
            if counts[d] > 1:
                raise ValueError(f"at most one {d.name} axis")
        if counts[KvDim.HEAD_SIZE] + counts[KvDim.PAYLOAD] > 1:
            raise ValueError("at most one of HEAD_SIZE / PAYLOAD")
        if counts[KvDim.PAYLOAD] and dims[-1] != KvDim.PAYLOAD:
            raise ValueError("PAYLOAD must be the trailing axis")
        if counts[KvDim.OUTER] and sizes[dims.index(KvDim.OUTER)] not in (1, 2):
            raise ValueError("OUTER axis size must be 1 or 2")
        object.__setattr__(self, "dims", dims)
        object.__setattr__(self, "sizes", sizes)

    def position(self, d: KvDim) -> int | None:
        return self.dims.index(d) if d in self.dims else None

    def size_of(self, d: KvDim) -> int | None:
        i = self.position(d)
        return None if i is None else self.sizes[i]

    @property
    def total_elements(self) -> int:
        n = 1
        for s in self.sizes:
            n *= s
        return n

    @property
    def block_axis(self) -> int:
        return self.dims.index(KvDim.BLOCK)

    @property
    def outer_size(self) -> int:
        return self.size_of(KvDim.OUTER) or 1

    @property
    def page_size(self) -> int:
        p = self.size_of(KvDim.PAGE)
        if p is None:
            raise ValueError("layout has no PAGE axis")
        return p

    @property
    def head_count(self) -> int | None:
        return self.size_of(KvDim.HEAD)

    @property
    def head_size(self) -> int | None:
        return self.size_of(KvDim.HEAD_SIZE)

    @property
    def inner_elements(self) -> int | None:
        """Elements of one (block, layer, outer) chunk: page x heads x head_size (or payload)."""
        page = self.size_of(KvDim.PAGE)
        tail = self.size_of(KvDim.HEAD_SIZE) or self.size_of(KvDim.PAYLOAD)
        if page is None or tail is None:
            return None
        return page * (self.size_of(KvDim.HEAD) or 1) * tail

    def inner_bytes(self, dtype_bytes: int) -> int | None:
        n = self.inner_elements
        return None if n is None else n * dtype_bytes


@dataclass(frozen=True)
class KvDimStrides:
    byte_strides: tuple[int, ...]
    elem_size: int

    @classmethod
    def from_element_strides(cls, strides: Sequence[int], elem_size: int) -> "KvDimStrides":
        if elem_size <= 0:
            raise ValueError("elem_size must be positive")
        return cls(tuple(int(s) * elem_size for s in strides), elem_size)

    @classmethod
    def from_byte_strides(cls, strides: Sequence[int], elem_size: int) -> "KvDimStrides":
        if elem_size <= 0 or any(s % elem_size for s in strides):
            raise ValueError("byte strides must be multiples of the element size")
        return cls(tuple(int(s) for s in strides), elem_size)

    @classmethod
    def contiguous_for(cls, layout: KvDimLayout, elem_size: int) -> "KvDimStrides":
        out, acc = [], elem_size
        for s in reversed(layout.sizes):
            out.append(acc)
            acc *= s
        return cls(tuple(reversed(out)), elem_size)

    def contiguous_tail_bytes(self, layout: KvDimLayout) -> int:
        """Bytes of the longest trailing run of axes laid out densely (>= one element)."""
        if len(self.byte_strides) != len(layout.sizes):
            raise ValueError("stride rank differs from layout rank")
        run = self.elem_size
        for size, stride in zip(reversed(layout.sizes), reversed(self.byte_strides)):
            if size == 1:
                continue
            if stride != run:
                break
            run *= size
        return run

    def is_fully_contiguous(self, layout: KvDimLayout) -> bool:
        return self.contiguous_tail_bytes(layout) == layout.total_elements * self.elem_size


@dataclass(frozen=True)
class AxisSlice:
    """Window [start, start+len) of an axis of global length ``global_len``."""

    dim: KvDim
    start: int
    len: int
    global_len: int

    def __post_init__(self):
        if self.len <= 0 or self.start < 0 or self.start + self.len > self.global_len:
            raise ValueError(f"bad slice {self.start}+{self.len} of {self.global_len}")

    @classmethod
    def full(cls, dim: KvDim, global_len: int) -> "AxisSlice":
        return cls(dim, 0, global_len, global_len)

    @classmethod
    def shard(cls, dim: KvDim, rank: int, world: int, global_len: int) -> "AxisSlice":
        if world <= 0 or not 0 <= rank < world:
            raise ValueError(f"rank {rank} out of range for world {world}")
        if global_len % world:
            raise ValueError(f"{global_len} does not split evenly over {world} ranks")
        n = global_len // world
        return cls(dim, rank * n, n, global_len)

    @property
    def end(self) -> int:
        return self.start + self.len

    @property
    def is_full(self) -> bool:
        return self.start == 0 and self.len == self.global_len


@dataclass(frozen=True)
class AxisExtent:
    local: int
    global_: int
    start: int = 0

    @classmethod
    def full(cls, size: int) -> "AxisExtent":
        return cls(size, size, 0)

    @classmethod
    def from_slice(cls, s: AxisSlice) -> "AxisExtent":
        return cls(s.len, s.global_len, s.start)

    @property
    def is_full(self) -> bool:
        return self.start == 0 and self.local == self.global_


@dataclass(frozen=True)
class AxisIntersection:
    dim: KvDim
    src_local: range
    dst_local: range

    def __len__(self) -> int:
        return len(self.src_local)


def intersect_axis(src: AxisSlice, dst: AxisSlice) -> AxisIntersection | None:
    """Overlap of two windows of the same axis, in each side's local coordinates (None if disjoint)."""
    if src.dim != dst.dim:
        raise ValueError(f"axis mismatch: {src.dim} vs {dst.dim}")
    if src.global_len != dst.global_len:
        raise ValueError(f"{src.dim.name}: global lengths differ ({src.global_len} vs {dst.global_len})")
    lo, hi = max(src.start, dst.start), min(src.end, dst.end)
    if hi <= lo:
        return None
    return AxisIntersection(src.dim, range(lo - src.start, hi - src.start), range(lo - dst.start, hi - dst.start))


@dataclass(frozen=True)
class LayoutSignature:
    axes: tuple[tuple[KvDim, AxisExtent], ...]
    byte_strides: tuple[int, ...]
    elem_size: int
    region_axis: KvDim | None = None  # an axis whose index picks a separate allocation (layer-separate pools)

    def compatible(self, other: "LayoutSignature") -> bool:
        """Same labelled axes and global extents (strides and local windows may differ)."""
        return ([(d, e.global_) for d, e in self.axes] == [(d, e.global_) for d, e in other.axes]
                and self.elem_size == other.elem_size)


@dataclass
class CoordByLabel:
    """A coordinate addressed by axis label rather than position."""

    values: dict[KvDim, int] = field(default_factory=dict)

    def with_(self, d: KvDim, v: int) -> "CoordByLabel":
        self.values[d] = v
        return self

    def get(self, d: KvDim) -> int | None:
        return self.values.get(d)

    def has(self, d: KvDim) -> bool:
        return d in self.values

    def offset(self, layout: KvDimLayout, strides: KvDimStrides) -> int:
        """Byte offset of this coordinate (missing labels are 0)."""
        off = 0
        for d, s, st in zip(layout.dims, layout.sizes, strides.byte_strides):
            v = self.values.get(d, 0)
            if not 0 <= v < s:
                raise IndexError(f"{d.name}={v} outside [0, {s})")
            off += v * st
        return off


@dataclass(frozen=True)
class CanonicalBlockShape:
    """Per-block geometry two layouts must agree on before a transfer."""

    num_layers: int
    outer_dim: int
    page_size: int
    num_heads: int
    head_size: int
    dtype_bytes: int

    def require_equal(self, other: "CanonicalBlockShape") -> None:
        if self != other:
            diff = [k for k in self.__dataclass_fields__ if getattr(self, k) != getattr(other, k)]
            raise ValueError(f"block shapes differ in {diff}: {self} vs {other}")
