"""Label the axes of a serving framework's KV-cache tensors.

Attention backends disagree on KV tensor layout: flash-attn uses
``[2, num_blocks, block_size, heads, head_dim]`` per layer, flashinfer
``[num_blocks, 2, block_size, heads, head_dim]``, some backends put heads
before tokens (HND), cross-layer caches add a layer axis. Calling the
backend's shape function with pairwise-distinct prime sentinels for every
dimension reveals which axis is which; :func:`derive_block_layout` turns the
labels into a :class:`~kvbm_b200.physical.layout.KvLayout` description.

Parity: python/kvbm/vllm/dim_probe.py:39-476 (KvDim, prime sentinels :71-74,
probe_kv_dim_layout :90, derive_block_layout :198, build_dim_layout_from_tensor
:402) and crates/kvbm-common/src/tensor.rs (KvDim labels).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch

from ..common.tensor import KvDim
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig


# pairwise-distinct primes, none equal to 1 or 2 (2 is the K/V outer size)
SENTINELS = {KvDim.BLOCK: 1009, KvDim.PAGE: 17, KvDim.HEAD: 13, KvDim.HEAD_SIZE: 127, KvDim.LAYER: 23}


def probe_kv_dim_layout(shape_fn: Callable[[int, int, int, int], Sequence[int]],
                        with_layers: bool = False) -> list[KvDim]:
    """Label each axis of ``shape_fn(num_blocks, block_size, num_kv_heads, head_size)``."""
    s = SENTINELS
    shape = list(shape_fn(s[KvDim.BLOCK], s[KvDim.PAGE], s[KvDim.HEAD], s[KvDim.HEAD_SIZE]))
    inv = {v: k for k, v in s.items()}
    labels = []
    for d in shape:
        if d == 2:
            labels.append(KvDim.OUTER)
        elif d in inv:
            labels.append(inv[d])
        elif d == s[KvDim.HEAD] * s[KvDim.HEAD_SIZE]:
            labels.extend([KvDim.HEAD, KvDim.HEAD_SIZE])
        else:
            raise ValueError(f"cannot label axis of size {d} in {shape}")
    return labels


@dataclass
class DimLayout:
    labels: list[KvDim]
    cross_layer: bool

    @property
    def block_first(self) -> bool:
        order = [l for l in self.labels if l in (KvDim.BLOCK, KvDim.OUTER)]
        return order[0] == KvDim.BLOCK if order else True

    @property
    def inner(self) -> KvBlockLayout:
        p, h = self.labels.index(KvDim.PAGE), self.labels.index(KvDim.HEAD)
        return KvBlockLayout.OPERATIONAL_NHD if p < h else KvBlockLayout.OPERATIONAL_HND


def derive_block_layout(labels: Sequence[KvDim]) -> DimLayout:
    labels = list(labels)
    if labels[-1] != KvDim.HEAD_SIZE:
        raise ValueError("head_size must be the innermost axis")
    need = {KvDim.BLOCK, KvDim.PAGE, KvDim.HEAD, KvDim.HEAD_SIZE}
    if not need.issubset(labels):
        raise ValueError(f"missing axes in {labels}")
    return DimLayout(labels, KvDim.LAYER in labels)


def infer_from_shape(shape: Sequence[int], num_blocks: int, block_size: int, num_kv_heads: int,
                     head_size: int, num_layers: int | None = None) -> list[KvDim]:
    """Label a concrete tensor shape from known sizes (ambiguities resolved by vLLM conventions)."""
    sizes = {KvDim.BLOCK: num_blocks, KvDim.PAGE: block_size, KvDim.HEAD: num_kv_heads, KvDim.HEAD_SIZE: head_size}
    if num_layers:
        sizes[KvDim.LAYER] = num_layers
    labels: list[KvDim | None] = [None] * len(shape)
    labels[-1] = KvDim.HEAD_SIZE
    pref = [KvDim.BLOCK, KvDim.LAYER, KvDim.PAGE, KvDim.HEAD]
    used = {KvDim.HEAD_SIZE}
    for i, d in enumerate(shape[:-1]):
        layer_here = (sizes.get(KvDim.LAYER) == d and KvDim.LAYER not in used and i > 0
                      and labels[i - 1] == KvDim.BLOCK)  # cross-layer caches are [blocks, layers, ...]
        if (d == 2 and not layer_here and KvDim.OUTER not in used
                and (i == 0 or labels[i - 1] in (KvDim.BLOCK, KvDim.LAYER))):
            labels[i] = KvDim.OUTER
            used.add(KvDim.OUTER)
            continue
        for k in pref:
            if k not in used and sizes.get(k) == d:
                labels[i] = k
                used.add(k)
                break
        if labels[i] is None and d == 2 and KvDim.OUTER not in used:
            labels[i] = KvDim.OUTER
            used.add(KvDim.OUTER)
    if any(l is None for l in labels):
        raise ValueError(f"cannot label shape {tuple(shape)}")
    return labels  # type: ignore[return-value]


def layout_from_layer_tensors(tensors: list[torch.Tensor], labels: Sequence[KvDim], num_blocks: int, block_size: int,
                              num_kv_heads: int, head_size: int) -> KvLayout:
    dl = derive_block_layout(labels)
    cfg = LayoutConfig.for_model(num_blocks, len(tensors), num_kv_heads, head_size, block_size, tensors[0].dtype,
                                 outer_dim=2 if KvDim.OUTER in labels else 1)
    return KvLayout.over_layer_tensors(cfg, tensors, block_layout=dl.inner, block_first=dl.block_first)


def layout_from_cross_layer_tensor(t: torch.Tensor, labels: Sequence[KvDim], block_size: int, num_kv_heads: int,
                                   head_size: int) -> KvLayout:
    dl = derive_block_layout(labels)
    if labels[0] != KvDim.BLOCK or labels[1] != KvDim.LAYER:
        raise ValueError("cross-layer caches must be [blocks, layers, ...]")
    nb, nl = t.shape[0], t.shape[1]
    cfg = LayoutConfig.for_model(nb, nl, num_kv_heads, head_size, block_size, t.dtype,
                                 outer_dim=2 if KvDim.OUTER in labels else 1)
    return KvLayout.over_tensor(cfg, t, "fully_contiguous", dl.inner)
