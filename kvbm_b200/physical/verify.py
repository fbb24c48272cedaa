"""Verification and calibration utilities for KV pools.

* :func:`checksum_blocks` - per-block 64-bit checksums computed on the GPU
  (``kvbm_kv_checksum``) for device and mapped-pinned pools, or on the host
  for CPU pools. The value depends on the block's contents in canonical
  ``[layer, outer, token, head, dim]`` order only, so a block hashes equal
  before and after a transfer between pools of different physical layouts.
* :func:`checksum_reference` - the same function in numpy (the definition).
* :func:`fill_blocks` - deterministic fill patterns for tests and benchmarks.
* :class:`StartupBenchmark` - measures the copy engines for a (src, dst)
  layout pair once, caches the result on disk keyed by device and layout
  signature, and tells the transfer manager which engine to use when
  ``TransferCapabilities.startup_benchmark`` is on.

Parity: crates/kvbm-physical/src/transfer/{checksum.rs:43,66 (per-block /
per-layer BLAKE3 checksums), fill.rs:28-134 (fill patterns),
benchmark.rs:86-412 (startup benchmark cache)}. The checksum is a
splitmix64-mixed word sum instead of BLAKE3 so that it reduces in parallel
on the GPU and is independent of the physical layout.
"""

from __future__ import annotations

import enum
import hashlib
import json
import os
import threading
from pathlib import Path

import numpy as np
import torch

from .layout import KvLayout
from .memory import NumaHostBuffer, PinnedBuffer, SharedPinnedBuffer

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def checksum_reference(canonical: np.ndarray | torch.Tensor) -> int:
    """Checksum of one block given as canonical ``[layers, outer, page, heads, dim]`` values.

    Sum (mod 2^64) over the block's 4-byte words ``w`` (in canonical order,
    index ``i``) of ``mix64((i << 32) ^ w ^ 0x9e3779b97f4a7c15)`` with
    mix64 the splitmix64 finalizer.
    """
    if isinstance(canonical, torch.Tensor):
        t = canonical.detach().cpu().contiguous()
        raw = t.view(torch.uint8).numpy() if t.dtype != torch.uint8 else t.numpy()
    else:
        raw = np.ascontiguousarray(canonical).view(np.uint8)
    words = raw.reshape(-1).view(np.uint32).astype(np.uint64)
    idx = np.arange(words.size, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = _mix64((idx << np.uint64(32)) ^ words ^ _GOLD)
        return int(h.sum(dtype=np.uint64))


def _device_readable(layout: KvLayout) -> bool:
    """True when kernels may read the pool: device / peer memory, or page-locked host memory."""
    if layout.location in ("device", "peer"):
        return True
    b = layout.backing
    if isinstance(b, torch.Tensor):
        return b.is_pinned()
    if isinstance(b, NumaHostBuffer):
        return b.pinned
    return isinstance(b, (PinnedBuffer, SharedPinnedBuffer))


def checksum_blocks(layout: KvLayout, ids, *, layer_begin: int = 0, num_layers: int | None = None) -> list[int]:
    """Per-block checksums of ``ids`` (see :func:`checksum_reference`)."""
    ids = [int(i) for i in ids]
    if _device_readable(layout) and torch.cuda.is_available():
        from ..ops import kv_ops

        out = kv_ops.kv_checksum(layout, ids, layer_begin=layer_begin, num_layers=num_layers)
        return [v & ((1 << 64) - 1) for v in out.cpu().tolist()]
    nl = layout.config.num_layers - layer_begin if num_layers is None else num_layers
    blocks = layout.gather_blocks(ids)[:, layer_begin:layer_begin + nl]
    return [checksum_reference(b) for b in blocks]


class FillPattern(enum.Enum):
    ZEROS = "zeros"
    CONSTANT = "constant"      # every element = value
    BLOCK_ID = "block_id"      # every element of block b = (b % 251) + 1
    INDEX = "index"            # element = f(block, layer, outer, token, head, dim), exact in bf16/fp16
    RANDOM = "random"          # seeded normal values


def _canonical_pattern(layout: KvLayout, ids: list[int], pattern: FillPattern, value: float, seed: int):
    c = layout.config
    shape = (len(ids), c.num_layers, c.outer_dim, c.page_size, c.num_heads, c.head_dim)
    dt = torch.float32
    if pattern == FillPattern.ZEROS:
        return torch.zeros(shape, dtype=dt)
    if pattern == FillPattern.CONSTANT:
        return torch.full(shape, float(value), dtype=dt)
    if pattern == FillPattern.BLOCK_ID:
        b = torch.tensor([(i % 251) + 1 for i in ids], dtype=dt)
        return b.view(-1, 1, 1, 1, 1, 1).expand(shape).clone()
    if pattern == FillPattern.INDEX:
        # small integers (< 256) so the values are exact in every 16-bit dtype
        g = [torch.arange(n, dtype=torch.int64) for n in shape]
        g[0] = torch.tensor(ids, dtype=torch.int64)
        acc = torch.zeros(shape, dtype=torch.int64)
        for k, (ax, mul) in enumerate(zip(g, (7, 5, 3, 11, 13, 1))):
            view = [1] * 6
            view[k] = -1
            acc += ax.view(view) * mul
        return (acc % 251).to(dt)
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=gen, dtype=dt)


def fill_blocks(layout: KvLayout, ids, pattern: FillPattern | str = FillPattern.INDEX, value: float = 1.0,
                seed: int = 0) -> None:
    """Write a deterministic pattern into blocks ``ids`` (any pool location, any layout)."""
    ids = [int(i) for i in ids]
    if not ids:
        return
    vals = _canonical_pattern(layout, ids, FillPattern(pattern), value, seed)
    if layout.dtype == torch.float8_e4m3fn:
        data = vals.to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        data = vals.to(layout.dtype)
    layout.scatter_blocks(ids, data)


class StartupBenchmark:
    """Measure transfer engines for a layout pair once; cache the winner on disk."""

    ENGINES = ("tile", "tma", "pairs", "ce")

    def __init__(self, cache_path: str | os.PathLike | None = None, blocks: int = 64, iters: int = 5):
        self.path = Path(cache_path or os.environ.get("KVBM_BENCH_CACHE",
                                                      Path.home() / ".cache" / "kvbm" / "startup_bench.json"))
        self.blocks, self.iters = blocks, iters
        self._lock = threading.Lock()
        self._cache: dict[str, dict] = {}
        if self.path.exists():
            try:
                self._cache = json.loads(self.path.read_text())
            except (OSError, ValueError):
                self._cache = {}

    @staticmethod
    def key(src: KvLayout, dst: KvLayout) -> str:
        dev = torch.cuda.get_device_name() if torch.cuda.is_available() else "cpu"
        sig = []
        for l in (src, dst):
            c = l.config
            sig.append((l.location, l.kind, l.block_layout.name, str(l.dtype), c.num_layers, c.outer_dim,
                        c.page_size, c.num_heads, c.head_dim))
        return hashlib.sha256(json.dumps([dev, sig]).encode()).hexdigest()[:24]

    def lookup(self, src: KvLayout, dst: KvLayout) -> str | None:
        r = self._cache.get(self.key(src, dst))
        return r["best"] if r else None

    def record(self, src: KvLayout, dst: KvLayout, gbps: dict[str, float]) -> str:
        best = max(gbps, key=gbps.get)
        with self._lock:
            self._cache[self.key(src, dst)] = {"best": best, "gbps": gbps}
            self.path.parent.mkdir(parents=True, exist_ok=True)
            tmp = self.path.with_suffix(".tmp")
            tmp.write_text(json.dumps(self._cache, indent=1))
            os.replace(tmp, self.path)
        return best

    def run(self, manager, src_handle: int, dst_handle: int) -> str:
        """Time each engine on ``blocks`` block pairs (CUDA events) and cache the fastest."""
        from .transfer import TransferOptions

        src, dst = manager.layout(src_handle).layout, manager.layout(dst_handle).layout
        cached = self.lookup(src, dst)
        if cached is not None:
            return cached
        n = min(self.blocks, src.config.num_blocks, dst.config.num_blocks)
        ids = list(range(n))
        nbytes = n * src.config.bytes_per_block
        gbps: dict[str, float] = {}
        for eng in self.ENGINES:
            try:
                opts = TransferOptions(engine=eng)
                manager.execute_transfer(src_handle, ids, dst_handle, ids, opts).wait()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                s.record()
                for _ in range(self.iters):
                    manager.execute_transfer(src_handle, ids, dst_handle, ids, opts).wait()
                e.record()
                e.synchronize()
                gbps[eng] = nbytes * self.iters / (s.elapsed_time(e) * 1e-3) / 1e9
            except (ValueError, RuntimeError):
                continue  # engine does not apply to this pair
        if not gbps:
            raise RuntimeError("no transfer engine applies to this layout pair")
        return self.record(src, dst, gbps)
