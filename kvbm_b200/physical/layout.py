"""Physical KV layouts: how (block, layer, outer, token, head, dim) maps to bytes.

A :class:`KvLayout` is a strided description of one KV pool:

* ``fully_contiguous`` (FC): one region, ``[num_blocks, num_layers, outer, ...]``
  with the per-chunk inner order NHD ``[page, heads, head_dim]`` or HND
  ``[heads, page, head_dim]``, or the universal block order
  ``[num_blocks, heads, num_layers, outer, page, head_dim]``;
* ``layer_separate`` (LW): one region per layer, block-first
  ``[num_blocks, outer, page, heads, head_dim]`` or outer-first
  ``[outer, num_blocks, page, heads, head_dim]`` (vLLM's flash-attn layout).

Every layout reduces to per-layer base addresses plus byte strides for
block, outer, token and head, which is exactly what the sm_100a transfer
kernels consume (``KvbmSide`` in ``kvbm_kernels.h``). A layout can be
exported as a :class:`LayoutDescriptor` (plain data + one CUDA IPC handle)
and re-materialised in another process on top of the mapped pool.

Parity: crates/kvbm-physical/src/layout/{config.rs:15-76, fully_contiguous.rs,
layer_separate.rs, serialize.rs}, crates/kvbm-common/src/block.rs:46-140
(KvBlockLayout and requires_transform).
"""

from __future__ import annotations

import enum
from dataclasses import asdict, dataclass, field

import torch

from ..ops import _lib
from .memory import (DeviceBuffer, NumaHostBuffer, PeerBuffer, PinnedBuffer, SharedHostBuffer, SharedPinnedBuffer,
                     gpu_numa_node)

DTYPE_CODE = {
    torch.float16: _lib.F16,
    torch.bfloat16: _lib.BF16,
    torch.float32: _lib.F32,
    torch.float64: _lib.F64,
    torch.float8_e4m3fn: _lib.FP8_E4M3,
}
DTYPE_NAME = {
    torch.float16: "float16",
    torch.bfloat16: "bfloat16",
    torch.float32: "float32",
    torch.float64: "float64",
    torch.float8_e4m3fn: "float8_e4m3fn",
}
NAME_DTYPE = {v: k for k, v in DTYPE_NAME.items()}


class KvBlockLayout(str, enum.Enum):
    """Order of the permutable dims inside a block (head_dim always innermost)."""

    UNIVERSAL = "universal"            # [nh, nl, no, nt, hd]
    OPERATIONAL_NHD = "operational_nhd"  # [nl, no, nt, nh, hd]
    OPERATIONAL_HND = "operational_hnd"  # [nl, no, nh, nt, hd]
    UNKNOWN = "unknown"

    def dim_order(self):
        return {
            KvBlockLayout.UNIVERSAL: ("head", "layer", "outer", "page"),
            KvBlockLayout.OPERATIONAL_HND: ("layer", "outer", "head", "page"),
            KvBlockLayout.OPERATIONAL_NHD: ("layer", "outer", "page", "head"),
        }.get(self)

    def requires_transform(self, other: "KvBlockLayout") -> bool:
        a, b = self.dim_order(), other.dim_order()
        if a is None and b is None:
            return False
        return a != b


def _is_pow2(x: int) -> bool:
    return x > 0 and (x & (x - 1)) == 0


@dataclass(frozen=True)
class LayoutConfig:
    """Geometry of a KV pool (field names follow the reference's LayoutConfig)."""

    num_blocks: int
    num_layers: int
    outer_dim: int
    page_size: int
    inner_dim: int  # page_size * num_heads * head_dim
    alignment: int = 1
    dtype_width_bytes: int = 2
    num_heads: int | None = None
    dtype: str | None = None

    def validate(self) -> None:
        if self.num_blocks < 1 or self.num_layers < 1 or self.inner_dim < 1:
            raise ValueError("num_blocks, num_layers and inner_dim must be >= 1")
        if self.outer_dim not in (1, 2):
            raise ValueError("outer_dim must be 1 or 2")
        if not _is_pow2(self.page_size):
            raise ValueError("page_size must be a positive power of two")
        if not _is_pow2(self.alignment):
            raise ValueError("alignment must be a power of two")
        if self.dtype_width_bytes not in (1, 2, 4, 8):
            raise ValueError("dtype_width_bytes must be 1, 2, 4 or 8")
        if self.num_heads is not None and self.inner_dim % (self.page_size * self.num_heads) != 0:
            raise ValueError("inner_dim must be divisible by page_size * num_heads")

    @property
    def head_dim(self) -> int:
        if self.num_heads is None:
            raise ValueError("num_heads is required for per-head addressing")
        return self.inner_dim // (self.page_size * self.num_heads)

    @property
    def torch_dtype(self) -> torch.dtype:
        if self.dtype is not None:
            return NAME_DTYPE[self.dtype]
        return {1: torch.float8_e4m3fn, 2: torch.bfloat16, 4: torch.float32, 8: torch.float64}[self.dtype_width_bytes]

    @property
    def bytes_per_chunk(self) -> int:
        """Bytes of one (block, layer, outer) chunk."""
        return self.inner_dim * self.dtype_width_bytes

    @property
    def bytes_per_block(self) -> int:
        return self.num_layers * self.outer_dim * self.bytes_per_chunk

    @classmethod
    def for_model(cls, num_blocks: int, num_layers: int, num_kv_heads: int, head_dim: int, page_size: int = 16,
                  dtype: torch.dtype = torch.bfloat16, outer_dim: int = 2) -> "LayoutConfig":
        width = torch.empty((), dtype=dtype).element_size()
        return cls(num_blocks=num_blocks, num_layers=num_layers, outer_dim=outer_dim, page_size=page_size,
                   inner_dim=page_size * num_kv_heads * head_dim, dtype_width_bytes=width, num_heads=num_kv_heads,
                   dtype=DTYPE_NAME[dtype])


@dataclass
class LayoutDescriptor:
    """Serializable description of a pool, enough to rebuild it in a peer process."""

    config: dict
    kind: str
    block_layout: str
    layer_offsets: list[int]
    block_stride: int
    outer_stride: int
    token_stride: int
    head_stride: int
    nbytes: int
    scales_offset: int | None = None
    ipc_handle: bytes | None = None
    device: int = 0
    extra: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["ipc_handle"] = self.ipc_handle.hex() if self.ipc_handle else None
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "LayoutDescriptor":
        d = dict(d)
        if d.get("ipc_handle"):
            d["ipc_handle"] = bytes.fromhex(d["ipc_handle"])
        return cls(**d)


class KvLayout:
    """Strided KV pool description over one backing region."""

    def __init__(self, config: LayoutConfig, kind: str, block_layout: KvBlockLayout, base_ptr: int,
                 layer_offsets: list[int], block_stride: int, outer_stride: int, token_stride: int,
                 head_stride: int, nbytes: int, location: str, device: int | None, backing=None,
                 scales_offset: int | None = None):
        config.validate()
        self.config = config
        self.kind = kind
        self.block_layout = block_layout
        self.base_ptr = int(base_ptr)
        self.layer_offsets = list(layer_offsets)
        self.block_stride = int(block_stride)
        self.outer_stride = int(outer_stride)
        self.token_stride = int(token_stride)
        self.head_stride = int(head_stride)
        self.nbytes = int(nbytes)
        self.location = location
        self.device = device
        self.backing = backing
        self.scales_offset = scales_offset
        self._flat_cache: torch.Tensor | None = None

    # ------------------------------------------------------------------ build
    @staticmethod
    def _strides(cfg: LayoutConfig, kind: str, block_layout: KvBlockLayout, block_first: bool = True):
        """Returns (layer_offsets, block_stride, outer_stride, token_stride, head_stride, data_bytes)."""
        e = cfg.dtype_width_bytes
        H = cfg.num_heads
        D = cfg.head_dim
        T, O, L, B = cfg.page_size, cfg.outer_dim, cfg.num_layers, cfg.num_blocks
        row = D * e
        if block_layout == KvBlockLayout.OPERATIONAL_HND:
            ts, hs = row, T * row
        else:
            ts, hs = H * row, row
        chunk = T * H * row
        if kind == "fully_contiguous":
            if block_layout == KvBlockLayout.UNIVERSAL:
                ts, hs = row, L * O * T * row
                layer_off = [l * O * T * row for l in range(L)]
                return layer_off, H * L * O * T * row, T * row, ts, hs, B * H * L * O * T * row
            layer_off = [l * O * chunk for l in range(L)]
            return layer_off, L * O * chunk, chunk, ts, hs, B * L * O * chunk
        if kind == "layer_separate":
            if block_layout == KvBlockLayout.UNIVERSAL:
                raise ValueError("universal block layout requires a fully contiguous pool")
            per_layer = B * O * chunk
            layer_off = [l * per_layer for l in range(L)]
            if block_first:
                return layer_off, O * chunk, chunk, ts, hs, L * per_layer
            return layer_off, chunk, B * chunk, ts, hs, L * per_layer
        raise ValueError(f"unknown layout kind {kind!r}")

    @classmethod
    def allocate(cls, config: LayoutConfig, kind: str = "fully_contiguous",
                 block_layout: KvBlockLayout = KvBlockLayout.OPERATIONAL_NHD, location: str = "device",
                 block_first: bool = True, fp8_scales: bool = False, device: int | None = None,
                 zero: bool = False, shm_name: str | None = None, numa_node: int | str | None = None,
                 hugepages: bool = False) -> "KvLayout":
        """Allocate a pool. ``location``: ``device`` (HBM), ``pinned`` (page-locked
        host memory mapped for the GPU) or ``shared`` (a named ``/dev/shm`` file
        other processes on the node can map; page-locked when CUDA is present).

        For ``pinned`` pools, ``numa_node`` places the memory on a NUMA node
        (``"gpu"``: the node nearest to the current GPU), optionally on 2 MiB
        ``hugepages``; by default ``cudaHostAlloc`` places it."""
        layer_off, bs, os_, ts, hs, data_bytes = cls._strides(config, kind, block_layout, block_first)
        scales_offset = None
        total = data_bytes
        if fp8_scales:
            scales_offset = (data_bytes + 255) // 256 * 256
            total = scales_offset + config.num_blocks * config.num_layers * config.outer_dim * config.num_heads * 4
        if location == "device":
            buf = DeviceBuffer(total, device=device, zero=zero)
            base = buf.ptr
            dev = buf.device
        elif location == "pinned" and (numa_node is not None or hugepages):
            node = gpu_numa_node(device) if numa_node in (None, "gpu") else int(numa_node)
            buf = NumaHostBuffer(total, node=node, hugepages=hugepages)  # zero-filled by first touch
            base = buf.device_ptr or buf.ptr
            dev = None
        elif location == "pinned":
            buf = PinnedBuffer(total)
            if zero:
                buf.tensor().zero_()
            base = buf.device_ptr
            dev = None
        elif location == "shared":
            import os
            import uuid

            name = shm_name or f"kvbm_g2_{os.getpid()}_{uuid.uuid4().hex[:8]}"
            buf = SharedPinnedBuffer(name, total) if torch.cuda.is_available() else SharedHostBuffer(name, total)
            # a new file reads as zeros
            base = getattr(buf, "device_ptr", buf.ptr)
            dev = None
            location = "pinned"
        else:
            raise ValueError("location must be 'device', 'pinned' or 'shared'")
        lay = cls(config, kind, block_layout, base, layer_off, bs, os_, ts, hs, total, location, dev, buf,
                  scales_offset)
        lay._block_first = block_first
        return lay

    @classmethod
    def over_tensor(cls, config: LayoutConfig, tensor: torch.Tensor, kind: str = "fully_contiguous",
                    block_layout: KvBlockLayout = KvBlockLayout.OPERATIONAL_NHD,
                    block_first: bool = True) -> "KvLayout":
        """Describe an existing contiguous tensor (e.g. a framework-owned KV cache)."""
        if not tensor.is_contiguous():
            raise ValueError("tensor must be contiguous")
        layer_off, bs, os_, ts, hs, data_bytes = cls._strides(config, kind, block_layout, block_first)
        nbytes = tensor.numel() * tensor.element_size()
        if nbytes < data_bytes:
            raise ValueError(f"tensor holds {nbytes} bytes, layout needs {data_bytes}")
        loc = "device" if tensor.is_cuda else "pinned"
        lay = cls(config, kind, block_layout, tensor.data_ptr(), layer_off, bs, os_, ts, hs, data_bytes, loc,
                  tensor.device.index if tensor.is_cuda else None, tensor)
        lay._block_first = block_first
        return lay

    @classmethod
    def over_layer_tensors(cls, config: LayoutConfig, tensors: list[torch.Tensor],
                           block_layout: KvBlockLayout = KvBlockLayout.OPERATIONAL_NHD,
                           block_first: bool = True) -> "KvLayout":
        """Describe per-layer tensors (layer-separate, one allocation per layer)."""
        if len(tensors) != config.num_layers:
            raise ValueError("one tensor per layer expected")
        _, bs, os_, ts, hs, _ = cls._strides(config, "layer_separate", block_layout, block_first)
        # per-layer allocations may sit in any address order: offsets are taken
        # from the lowest one so they are never negative
        base = min(t.data_ptr() for t in tensors)
        offsets = [t.data_ptr() - base for t in tensors]
        end = max(t.data_ptr() + t.numel() * t.element_size() for t in tensors)
        lay = cls(config, "layer_separate", block_layout, base, offsets, bs, os_, ts, hs, end - base,
                  "device" if tensors[0].is_cuda else "pinned",
                  tensors[0].device.index if tensors[0].is_cuda else None, tensors)
        lay._block_first = block_first
        lay._layer_tensors = tensors
        return lay

    # -------------------------------------------------------------- export
    def _framework_tensors(self) -> list[torch.Tensor] | None:
        """The framework-owned CUDA tensors this layout describes (one per layer, or one), else None."""
        ts = getattr(self, "_layer_tensors", None)
        if ts is None and isinstance(self.backing, torch.Tensor):
            ts = [self.backing]
        if ts and all(isinstance(t, torch.Tensor) and t.is_cuda for t in ts):
            return list(ts)
        return None

    def descriptor(self, with_ipc: bool = True) -> LayoutDescriptor:
        """A serialisable description of the pool. With ``with_ipc`` it also carries what
        another process needs to map the memory: the CUDA IPC handle of a pool this
        library allocated, or, for a framework-owned KV cache (an inference engine's own
        tensors, described with ``over_tensor`` / ``over_layer_tensors``), one PyTorch
        CUDA IPC record per tensor (the allocation's handle, the tensor's offset in it,
        and PyTorch's cross-process reference count, which keeps the memory alive while a
        peer holds it)."""
        handle = None
        extra: dict = {}
        if with_ipc:
            if isinstance(self.backing, DeviceBuffer):
                handle = self.backing.ipc_handle()
            else:
                ts = self._framework_tensors()
                if ts is None:
                    raise ValueError("only device pools (allocated here or framework-owned CUDA tensors) can be "
                                     "exported")
                extra["torch_ipc"] = [_torch_ipc_export(t) for t in ts]
        cfg = asdict(self.config)
        return LayoutDescriptor(config=cfg, kind=self.kind, block_layout=self.block_layout.value,
                                layer_offsets=self.layer_offsets, block_stride=self.block_stride,
                                outer_stride=self.outer_stride, token_stride=self.token_stride,
                                head_stride=self.head_stride, nbytes=self.nbytes, scales_offset=self.scales_offset,
                                ipc_handle=handle, device=self.device or 0, extra=extra)

    @classmethod
    def from_descriptor(cls, desc: LayoutDescriptor, device: int | None = None) -> "KvLayout":
        """Map a peer's exported pool into this process (CUDA IPC; over NVLink when the
        pool is on another GPU)."""
        cfg = LayoutConfig(**desc.config)
        recs = (desc.extra or {}).get("torch_ipc")
        if recs:
            if device is not None:
                torch.cuda.set_device(device)
            ts = [_torch_ipc_import(r) for r in recs]
            if len(ts) == 1:
                base, offsets = ts[0].data_ptr(), list(desc.layer_offsets)
            else:  # one tensor per layer, each mapped wherever the driver put it
                base = min(t.data_ptr() for t in ts)
                offsets = [t.data_ptr() - base for t in ts]
            lay = cls(cfg, desc.kind, KvBlockLayout(desc.block_layout), base, offsets, desc.block_stride,
                      desc.outer_stride, desc.token_stride, desc.head_stride,
                      max(t.data_ptr() + t.numel() * t.element_size() for t in ts) - base, "peer",
                      torch.cuda.current_device(), ts, desc.scales_offset)
            return lay
        peer = PeerBuffer(desc.ipc_handle, desc.nbytes, device=device)
        lay = cls(cfg, desc.kind, KvBlockLayout(desc.block_layout), peer.ptr, desc.layer_offsets,
                  desc.block_stride, desc.outer_stride, desc.token_stride, desc.head_stride, desc.nbytes,
                  "peer", peer.device, peer, desc.scales_offset)
        return lay

    # -------------------------------------------------------------- access
    @property
    def dtype(self) -> torch.dtype:
        return self.config.torch_dtype

    @property
    def dtype_code(self) -> int:
        return DTYPE_CODE[self.dtype]

    @property
    def scales_ptr(self) -> int:
        return self.base_ptr + self.scales_offset if self.scales_offset is not None else 0

    def layer_base(self, layer: int) -> int:
        return self.base_ptr + self.layer_offsets[layer]

    def memory_region(self, block: int, layer: int, outer: int) -> tuple[int, int]:
        """Address and size of one (block, layer, outer) chunk, when contiguous."""
        if self.block_layout == KvBlockLayout.UNIVERSAL:
            raise ValueError("universal chunks are not contiguous per (layer, outer)")
        return (self.layer_base(layer) + block * self.block_stride + outer * self.outer_stride,
                self.config.bytes_per_chunk)

    def is_fully_contiguous_block(self) -> bool:
        return self.kind == "fully_contiguous"

    def side(self, ids: torch.Tensor | None, layer_begin: int = 0, num_layers: int | None = None,
             head_offset: int = 0) -> _lib.KvbmSide:
        """Kernel-side description for the given block ids (int32, device-accessible)."""
        n = self.config.num_layers - layer_begin if num_layers is None else num_layers
        if layer_begin < 0 or layer_begin + n > self.config.num_layers:
            raise ValueError("layer range out of bounds")
        if n > _lib.MAX_LAYERS:
            raise ValueError(f"at most {_lib.MAX_LAYERS} layers per launch")
        # the struct depends only on where the ids live, not on their values,
        # so repeated launches (one per layer in streaming transfers) reuse it
        key = (ids.data_ptr() if ids is not None else 0, layer_begin, n, head_offset)
        cache = self.__dict__.setdefault("_side_cache", {})
        hit = cache.get(key)
        if hit is not None:
            return hit
        if len(cache) > 4096:
            cache.clear()
        s = _lib.KvbmSide()
        s.mode = _lib.ADDR_LAYER_BASES
        s.head_offset = head_offset
        s.ids = ids.data_ptr() if ids is not None else None
        s.block_stride = self.block_stride
        s.outer_stride = self.outer_stride
        s.token_stride = self.token_stride
        s.head_stride = self.head_stride
        for i in range(n):
            s.layer_base[i] = self.layer_base(layer_begin + i)
        if self.scales_offset is not None:
            c = self.config
            s.scales = self.scales_ptr
            s.s_block = c.num_layers * c.outer_dim * c.num_heads
            s.s_layer = c.outer_dim * c.num_heads
            s.s_outer = c.num_heads
            s.s_head = 1
            s.s_layer_offset = layer_begin
        cache[key] = s
        return s

    # ------------------------------------------------- torch views (oracles)
    def _flat(self) -> torch.Tensor:
        if self._flat_cache is None:
            if self.location == "device":
                t = torch.as_tensor(_RawDev(self.base_ptr, self.nbytes), device=f"cuda:{self.device}")
            elif self.location == "pinned":
                if isinstance(self.backing, (PinnedBuffer, SharedHostBuffer, NumaHostBuffer)):
                    t = self.backing.tensor()
                else:
                    t = self.backing.view(torch.uint8).reshape(-1)
            else:
                raise ValueError("peer pools have no local torch view")
            self._flat_cache = t
        return self._flat_cache

    def layer_view(self, layer: int) -> torch.Tensor:
        """[num_blocks, outer, page, heads, head_dim] strided view of one layer."""
        c = self.config
        e = c.dtype_width_bytes
        flat = self._flat()
        # fp8 pools are viewed as raw bytes: indexing kernels do not cover float8
        typed = flat if self.dtype in (torch.uint8, torch.float8_e4m3fn) else flat.view(self.dtype)
        return torch.as_strided(
            typed,
            (c.num_blocks, c.outer_dim, c.page_size, c.num_heads, c.head_dim),
            (self.block_stride // e, self.outer_stride // e, self.token_stride // e, self.head_stride // e, 1),
            self.layer_offsets[layer] // e,
        )

    def scales_view(self) -> torch.Tensor | None:
        if self.scales_offset is None:
            return None
        c = self.config
        flat = self._flat()
        n = c.num_blocks * c.num_layers * c.outer_dim * c.num_heads
        return flat[self.scales_offset:self.scales_offset + n * 4].view(torch.float32).view(
            c.num_blocks, c.num_layers, c.outer_dim, c.num_heads)

    def gather_blocks(self, ids) -> torch.Tensor:
        """Canonical copy [n, layers, outer, page, heads, head_dim] of the given blocks."""
        ids_t = torch.as_tensor(ids, dtype=torch.long)
        outs = []
        for l in range(self.config.num_layers):
            v = self.layer_view(l)
            outs.append(v[ids_t.to(v.device)])
        return torch.stack(outs, dim=1)

    def scatter_blocks(self, ids, data: torch.Tensor) -> None:
        """Write canonical [n, layers, outer, page, heads, head_dim] data into the pool."""
        ids_t = torch.as_tensor(ids, dtype=torch.long)
        for l in range(self.config.num_layers):
            v = self.layer_view(l)
            v[ids_t.to(v.device)] = data[:, l].to(v.device)


class _RawDev:
    """__cuda_array_interface__ over a raw device range (no ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.ptr, self.nbytes = ptr, nbytes

    @property
    def __cuda_array_interface__(self):
        return {"shape": (self.nbytes,), "typestr": "|u1", "data": (self.ptr, False), "version": 3,
                "strides": None, "stream": None}


def _torch_ipc_export(t: torch.Tensor) -> dict:
    """PyTorch's CUDA IPC record of ``t`` as plain data (no pickle: the record crosses
    process boundaries through files other local users could write)."""
    from torch.multiprocessing.reductions import reduce_tensor

    _, a = reduce_tensor(t)
    (_, size, stride, offset, _, dtype, dev, handle, ssize, soff, _, rc_handle, rc_off, ev_handle, ev_sync) = a
    return {"size": list(size), "stride": list(stride), "offset": int(offset), "dtype": str(dtype).split(".")[-1],
            "device": int(dev), "handle": bytes(handle).hex(), "storage_bytes": int(ssize),
            "storage_offset": int(soff), "rc_handle": bytes(rc_handle).hex(), "rc_offset": int(rc_off),
            "event": bytes(ev_handle).hex() if ev_handle is not None else None, "event_sync": bool(ev_sync)}


def _torch_ipc_import(r: dict) -> torch.Tensor:
    from torch.multiprocessing.reductions import rebuild_cuda_tensor

    dtype = getattr(torch, r["dtype"])
    if not isinstance(dtype, torch.dtype):
        raise ValueError(f"bad dtype {r['dtype']!r} in an IPC record")
    return rebuild_cuda_tensor(torch.Tensor, torch.Size(r["size"]), tuple(r["stride"]), int(r["offset"]),
                               torch.storage.TypedStorage, dtype, int(r["device"]), bytes.fromhex(r["handle"]),
                               int(r["storage_bytes"]), int(r["storage_offset"]), False,
                               bytes.fromhex(r["rc_handle"]), int(r["rc_offset"]),
                               bytes.fromhex(r["event"]) if r.get("event") else None, bool(r["event_sync"]))
