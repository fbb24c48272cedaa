"""Python entry points of the KV transfer kernels (sm_100a, libkvbm_cuda.so).

All functions are asynchronous on the given (or current) CUDA stream and take
torch tensors / :class:`~kvbm_b200.physical.layout.KvLayout` pools. Block-id
tensors must be int32 and device-accessible.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


_upload_streams: dict[int, torch.cuda.Stream] = {}


def upload(host: torch.Tensor, device: torch.device, stream=None) -> torch.Tensor:
    """Copy a small host tensor (block ids, pointer tables) to ``device`` for use on ``stream``.

    The copy runs on a dedicated idle stream, so it does not wait behind the
    target stream's queued transfers (a pageable copy is synchronous with the
    work already in its stream) and needs no page-locked staging allocation;
    the target stream waits on an event for it.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    us = _upload_streams.get(idx)
    if us is None:
        us = _upload_streams[idx] = torch.cuda.Stream(device=idx)
    target = stream if isinstance(stream, torch.cuda.Stream) else torch.cuda.current_stream(idx)
    with torch.cuda.stream(us):
        d = host.to(device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(us)
    target.wait_event(ev)
    d.record_stream(target)
    return d


def _ids(ids, device, stream=None) -> torch.Tensor:
    if isinstance(ids, torch.Tensor) and ids.dtype == torch.int32 and (ids.is_cuda or ids.is_pinned()):
        return ids
    t = torch.as_tensor(ids, dtype=torch.int32)
    return upload(t, device, stream) if device is not None else t


ENGINE_CODES = {"auto": 0, "tile": 1, "tma": 2}
RAN_NAMES = {1: "tile", 2: "tma", 3: "tma_bulk"}
XFER_DST_LOCAL, XFER_BULK_PEER, XFER_NO_BULK = 1, 2, 4


def kv_transfer(src, src_ids, dst, dst_ids, *, layer_begin: int = 0, num_layers: int | None = None,
                dst_layer_begin: int | None = None, src_head_offset: int = 0, dst_head_offset: int = 0,
                num_heads: int | None = None, engine: str = "tile", max_ctas: int = 0, stream=None,
                bulk: bool | None = None) -> str:
    """Copy blocks ``src_ids`` of ``src`` into blocks ``dst_ids`` of ``dst``; returns the kernel that ran.

    Fuses, in one launch: the layout transform between the two pools (FC/LW,
    NHD/HND/universal), a KV-head slice (``num_heads`` heads starting at
    ``src_head_offset`` land at ``dst_head_offset``: heterogeneous-TP
    resharding), and fp8 e4m3 block-scaled quantisation or dequantisation when
    the pool dtypes differ. ``dst`` may be a peer GPU's pool mapped over
    NVLink (``KvLayout.from_descriptor``) or a pinned host pool (G2).

    ``engine``: ``"tile"`` (warp per head tile, direct 16-byte loads),
    ``"tma"`` (bulk async copies staged through shared memory; raises when
    the source chunks are not contiguous / aligned, never falls back) or
    ``"auto"`` (``"tma"`` when it can, else ``"tile"``). Among the TMA
    kernels, same-layout whole-chunk copies run as the bulk copy (TMA loads
    and TMA stores only) when the destination is this GPU's memory, or any
    memory when ``bulk`` is True (``bulk=False`` never uses it). Returns
    ``"tile"``, ``"tma"`` or ``"tma_bulk"``.
    """
    n_pairs = len(src_ids)
    if n_pairs != len(dst_ids):
        raise ValueError("src_ids and dst_ids differ in length")
    if engine not in ENGINE_CODES:
        raise ValueError(f"unknown transfer engine {engine!r}")
    if n_pairs == 0:
        return "none"
    sc, dc = src.config, dst.config
    nl = sc.num_layers - layer_begin if num_layers is None else num_layers
    dlb = layer_begin if dst_layer_begin is None else dst_layer_begin
    nh = num_heads if num_heads is not None else min(sc.num_heads - src_head_offset, dc.num_heads - dst_head_offset)
    if src_head_offset + nh > sc.num_heads or dst_head_offset + nh > dc.num_heads:
        raise ValueError("head slice out of range")
    if sc.head_dim != dc.head_dim or sc.page_size != dc.page_size or sc.outer_dim != dc.outer_dim:
        raise ValueError("pools differ in head_dim, page_size or outer_dim")
    dev = torch.device("cuda", torch.cuda.current_device())
    sid = _ids(src_ids, dev, stream)
    did = _ids(dst_ids, dev, stream)
    s = src.side(sid, layer_begin, nl, src_head_offset)
    d = dst.side(did, dlb, nl, dst_head_offset)
    shape = _lib.KvbmTileShape(n_pairs, nl, sc.outer_dim, nh, sc.page_size, sc.head_dim, src.dtype_code,
                               dst.dtype_code)
    lib = _lib.load()
    st = _stream(stream)
    if stream is not None and isinstance(stream, torch.cuda.Stream):
        # temporaries uploaded here are read by the kernel on `stream`
        for t in (sid, did):
            if t.is_cuda:
                t.record_stream(stream)
    flags = 0
    if bulk is False:
        flags |= XFER_NO_BULK
    elif bulk:
        flags |= XFER_BULK_PEER
    elif getattr(dst, "location", None) == "device" and (dst.device is None or dst.device == dev.index):
        flags |= XFER_DST_LOCAL
    ran = C.c_int(0)
    rc = lib.kvbm_kv_xfer(C.byref(s), C.byref(d), C.byref(shape), ENGINE_CODES[engine], max_ctas, flags,
                          C.byref(ran), st)
    if rc != 0 and engine == "tma":
        raise _lib.KvbmCudaError("kvbm_kv_xfer: the TMA engine cannot take this transfer (source chunks not "
                                 "contiguous or not 16-byte aligned); use engine='auto' or 'tile'")
    _lib.check(rc, "kvbm_kv_xfer")
    _lib.count_launches(1 if ran.value else 0)
    return RAN_NAMES.get(ran.value, "none")


def transfer_status(reset: bool = False, device: int | None = None) -> int:
    """The TMA engines' status word for ``device`` (0: no error since the last reset;
    2: a misaligned chunk was refused; 3: a pipeline wait gave up). A host read of
    mapped memory: no device synchronization, so read it after the transfer's
    stream has passed the launch."""
    dev = torch.cuda.current_device() if device is None else device
    return int(_lib.load().kvbm_xfer_status(dev, 1 if reset else 0))


def check_transfer_status(device: int | None = None) -> None:
    """Raise (and clear the word) if a TMA transfer on ``device`` reported an error."""
    st = transfer_status(reset=True, device=device)
    if st:
        what = {2: "a chunk address was misaligned", 3: "a pipeline wait gave up (bulk copy did not land)"}
        raise _lib.KvbmCudaError(f"KV transfer failed on the device: status {st} ({what.get(st, 'unknown')})")


def set_pipeline_wait_limit_ns(ns: int) -> None:
    """Test hook: the TMA engines' pipeline wait limit for later launches (0: the default 2 s)."""
    _lib.load().kvbm_xfer_set_wait_limit_ns(int(ns))


def set_cast_pipeline(on: bool) -> None:
    """fp8 casts: the software-pipelined persistent kernel (default) or the one-tile-at-a-time kernel."""
    _lib.load().kvbm_xfer_set_cast_pipeline(1 if on else 0)


CAST_SOFTCONV_DEFAULT = (0, 1)  # (quantise, dequantise) quarters, the measured best on B200


def set_cast_softconv(quant_quarters: int | None = None, dequant_quarters: int | None = None) -> None:
    """Pipelined fp8 casts of bf16 data: how many quarters (0, 1, 2 or 4) of the conversions run on
    the integer / FMA pipes instead of the conversion instructions, per direction (None: the
    default); the bits are the same for finite values."""
    q = CAST_SOFTCONV_DEFAULT[0] if quant_quarters is None else int(quant_quarters)
    d = CAST_SOFTCONV_DEFAULT[1] if dequant_quarters is None else int(dequant_quarters)
    _lib.load().kvbm_xfer_set_cast_softconv(q, d)


def kv_checksum(layout, ids, *, layer_begin: int = 0, num_layers: int | None = None, head_offset: int = 0,
                num_heads: int | None = None, stream=None) -> torch.Tensor:
    """Layout-independent 64-bit checksum of each block in ``ids`` (int64 tensor on the device).

    Two blocks holding the same values hash equal whatever their pools'
    physical layouts; see ``physical.verify.checksum_reference`` for the
    definition. Works on device pools and on mapped pinned (G2) pools.
    """
    c = layout.config
    nl = c.num_layers - layer_begin if num_layers is None else num_layers
    nh = c.num_heads - head_offset if num_heads is None else num_heads
    dev = torch.device("cuda", torch.cuda.current_device())
    out = torch.empty(len(ids), dtype=torch.int64, device=dev)
    if len(ids) == 0:
        return out
    sid = _ids(ids, dev)
    side = layout.side(sid, layer_begin, nl, head_offset)
    shape = _lib.KvbmTileShape(len(ids), nl, c.outer_dim, nh, c.page_size, c.head_dim, layout.dtype_code,
                               layout.dtype_code)
    _lib.check(_lib.load().kvbm_kv_checksum(C.byref(side), C.byref(shape), C.c_void_p(out.data_ptr()),
                                            _stream(stream)), "kvbm_kv_checksum")
    _lib.count_launches(1)
    return out


def kv_transfer_sides(src_side, dst_side, shape, *, engine: str = "tile", max_ctas: int = 0, stream=None,
                      flags: int = 0) -> str:
    """Low-level launch with prebuilt ``KvbmSide`` / ``KvbmTileShape`` structs; returns the kernel that ran."""
    lib = _lib.load()
    ran = C.c_int(0)
    _lib.check(lib.kvbm_kv_xfer(C.byref(src_side), C.byref(dst_side), C.byref(shape), ENGINE_CODES[engine], max_ctas,
                                flags, C.byref(ran), _stream(stream)), "kvbm_kv_xfer")
    _lib.count_launches(1 if ran.value else 0)
    return RAN_NAMES.get(ran.value, "none")


def _ptr_align(ptrs: list[int], nbytes: int) -> int:
    a = 16
    for p in [*ptrs, nbytes]:
        while a > 1 and p % a:
            a >>= 1
    return a


def copy_pairs(src_ptrs, dst_ptrs, nbytes: int, *, align: int | None = None, max_ctas: int = 0,
               stream=None) -> None:
    """Batched copy of equal-size regions split by bytes across all SMs.

    ``src_ptrs``/``dst_ptrs`` are int64 device tensors (or lists, uploaded
    here). Regions may be device, mapped pinned host or peer memory.
    """
    dev = torch.device("cuda", torch.cuda.current_device())
    if not isinstance(src_ptrs, torch.Tensor):
        if align is None:
            align = _ptr_align(list(src_ptrs) + list(dst_ptrs), nbytes)
        src_ptrs = upload(torch.tensor(list(src_ptrs), dtype=torch.int64), dev, stream)
        dst_ptrs = upload(torch.tensor(list(dst_ptrs), dtype=torch.int64), dev, stream)
    if align is None:
        align = 16 if nbytes % 16 == 0 else 1
    _lib.call("kvbm_copy_pairs", src_ptrs.data_ptr(), dst_ptrs.data_ptr(), src_ptrs.numel(), nbytes, align,
              max_ctas, _stream(stream))


def memcpy_2d_ce(dst: int, dpitch: int, src: int, spitch: int, width: int, height: int, stream=None) -> None:
    """Copy-engine baseline for a strided batch of equal rows (one cudaMemcpy2DAsync)."""
    _lib.check(_lib.load().kvbm_memcpy_2d_async(dst, dpitch, src, spitch, width, height, _stream(stream)),
               "kvbm_memcpy_2d_async")


def memcpy_pairs_ce(src_ptrs: list[int], dst_ptrs: list[int], nbytes: int, stream=None) -> None:
    """Copy-engine baseline: one cudaMemcpyAsync per region."""
    n = len(src_ptrs)
    s = (C.c_uint64 * n)(*src_ptrs)
    d = (C.c_uint64 * n)(*dst_ptrs)
    _lib.call("kvbm_memcpy_pairs_ce", C.cast(s, C.c_void_p), C.cast(d, C.c_void_p), n, nbytes, _stream(stream))


def _dt(t: torch.dtype) -> int:
    from ..physical.layout import DTYPE_CODE

    return DTYPE_CODE[t]


def universal_from_block(universal_ptrs: torch.Tensor, block_ptrs: torch.Tensor, nh: int, nl: int, no: int, nt: int,
                         hd: int, dtype: torch.dtype, layout: int, nl_full: int | None = None, nl_offset: int = 0,
                         stream=None) -> None:
    """Block stack (nl*no chunk pointers per block) -> universal [nh, nl_full, no, nt, hd]."""
    nb = universal_ptrs.numel()
    _lib.call("kvbm_universal_from_block", universal_ptrs.data_ptr(), block_ptrs.data_ptr(), nb, nh, nl, no, nt, hd,
              nl if nl_full is None else nl_full, nl_offset, _dt(dtype), layout, _stream(stream))


def block_from_universal(universal_ptrs: torch.Tensor, block_ptrs: torch.Tensor, nh: int, nl: int, no: int, nt: int,
                         hd: int, dtype: torch.dtype, layout: int, nl_full: int | None = None, nl_offset: int = 0,
                         stream=None) -> None:
    """Universal [nh, nl_full, no, nt, hd] -> block stack."""
    nb = universal_ptrs.numel()
    _lib.call("kvbm_block_from_universal", universal_ptrs.data_ptr(), block_ptrs.data_ptr(), nb, nh, nl, no, nt, hd,
              nl if nl_full is None else nl_full, nl_offset, _dt(dtype), layout, _stream(stream))


def nhd_hnd_transpose(src_chunks: torch.Tensor, dst_chunks: torch.Tensor, nb: int, nl: int, no: int, nt: int,
                      nh: int, hd: int, dtype: torch.dtype, src_layout: int, stream=None) -> None:
    """Per chunk, swap [nt, nh, hd] <-> [nh, nt, hd]."""
    _lib.call("kvbm_nhd_hnd_transpose", src_chunks.data_ptr(), dst_chunks.data_ptr(), nb, nl, no, nt, nh, hd,
              _dt(dtype), src_layout, _stream(stream))


def signal_flag(flag_ptr: int, value: int, stream=None) -> None:
    _lib.call("kvbm_signal_flag", flag_ptr, value, _stream(stream))


def signal_flag_multicast(flag_mc: int, stream=None) -> None:
    """Add 1 to a u64 counter through its NVLink multicast address (every member's copy)."""
    _lib.call("kvbm_signal_multicast", flag_mc, _stream(stream))


def wait_flag(flag_ptr: int, expected: int, timeout_ns: int, status_ptr: int, stream=None) -> None:
    _lib.call("kvbm_wait_flag", flag_ptr, expected, timeout_ns, status_ptr, _stream(stream))


def signal_flag_payload(flag_ptr: int, value: int, payload_dst: int, payload_src: int, n_words: int,
                        stream=None) -> None:
    """Copy ``n_words`` u64 words to ``payload_dst`` (peer memory), then release-store the flag."""
    _lib.call("kvbm_signal_flag_payload", flag_ptr, value, payload_dst, payload_src, n_words, _stream(stream))


def wait_flags_all(flags_ptr: int, n: int, expected: int, timeout_ns: int, status_ptr: int, stream=None) -> None:
    """Block ``stream`` until all ``n`` u64 flags reach ``expected`` (bounded; status=1 on timeout)."""
    _lib.call("kvbm_wait_flags_all", flags_ptr, n, expected, timeout_ns, status_ptr, _stream(stream))


def sm_count() -> int:
    return _lib.load().kvbm_sm_count()
