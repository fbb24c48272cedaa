"""ctypes binding of ``libkvbm_cuda.so`` (the sm_100a kernel library).

The library is built in-tree by :mod:`kvbm_b200._build`. Loading fails loudly
when it is missing: there is no eager/PyTorch fallback for any kernel.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

from .. import _build

MAX_LAYERS = 128

F16, BF16, F32, F64, FP8_E4M3 = 0, 1, 2, 3, 4
NHD, HND = 0, 1
ADDR_LAYER_BASES, ADDR_BLOCK_TABLE, ADDR_CHUNK_TABLE = 0, 1, 2


class KvbmSide(C.Structure):
    _fields_ = [
        ("mode", C.c_int32),
        ("head_offset", C.c_int32),
        ("chunk_layers", C.c_int32),
        ("chunk_outer", C.c_int32),
        ("table", C.c_void_p),
        ("ids", C.c_void_p),
        ("block_stride", C.c_int64),
        ("layer_stride", C.c_int64),
        ("layer_offset", C.c_int64),
        ("outer_stride", C.c_int64),
        ("token_stride", C.c_int64),
        ("head_stride", C.c_int64),
        ("scales", C.c_void_p),
        ("s_block", C.c_int64),
        ("s_layer", C.c_int64),
        ("s_outer", C.c_int64),
        ("s_head", C.c_int64),
        ("s_layer_offset", C.c_int64),
        ("layer_base", C.c_uint64 * MAX_LAYERS),
    ]


class KvbmTileShape(C.Structure):
    _fields_ = [
        ("num_pairs", C.c_int32),
        ("num_layers", C.c_int32),
        ("num_outer", C.c_int32),
        ("num_heads", C.c_int32),
        ("page_size", C.c_int32),
        ("head_dim", C.c_int32),
        ("src_dtype", C.c_int32),
        ("dst_dtype", C.c_int32),
    ]


_lock = threading.Lock()
_lib: C.CDLL | None = None

_VP = C.c_void_p
_I64 = C.c_int64
_U64 = C.c_uint64
_I32 = C.c_int32
_INT = C.c_int
_F32 = C.c_float
_SZ = C.c_size_t

_SIGS = {
    "kvbm_kv_tile_xfer": (_INT, [C.POINTER(KvbmSide), C.POINTER(KvbmSide), C.POINTER(KvbmTileShape), _INT, _VP]),
    "kvbm_kv_chunk_xfer_tma": (_INT, [C.POINTER(KvbmSide), C.POINTER(KvbmSide), C.POINTER(KvbmTileShape), _INT, _VP]),
    "kvbm_kv_xfer": (_INT, [C.POINTER(KvbmSide), C.POINTER(KvbmSide), C.POINTER(KvbmTileShape), _INT, _INT, _INT,
                            C.POINTER(_INT), _VP]),
    "kvbm_xfer_status": (_INT, [_INT, _INT]),
    "kvbm_xfer_set_wait_limit_ns": (None, [_U64]),
    "kvbm_xfer_set_cast_pipeline": (None, [_INT]),
    "kvbm_xfer_set_cast_softconv": (None, [_INT, _INT]),
    "kvbm_copy_pairs": (_INT, [_VP, _VP, _U64, _U64, _INT, _INT, _VP]),
    "kvbm_universal_from_block": (_INT, [_VP, _VP, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _INT, _INT, _VP]),
    "kvbm_block_from_universal": (_INT, [_VP, _VP, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _INT, _INT, _VP]),
    "kvbm_nhd_hnd_transpose": (_INT, [_VP, _VP, _SZ, _SZ, _SZ, _SZ, _SZ, _SZ, _INT, _INT, _VP]),
    "kvbm_signal_flag": (_INT, [_VP, _U64, _VP]),
    "kvbm_wait_flag": (_INT, [_VP, _U64, _U64, _VP, _VP]),
    "kvbm_signal_flag_payload": (_INT, [_VP, _U64, _VP, _VP, _INT, _VP]),
    "kvbm_wait_flags_all": (_INT, [_VP, _INT, _U64, _U64, _VP, _VP]),
    "kvbm_signal_multicast": (_INT, [_U64, _VP]),
    "kvbm_kv_multicast": (_INT, [_VP, _VP, _INT, _U64, _I64, _I64, _I64, _INT, _VP, _VP, _INT, _INT, _U64, _VP, _VP,
                                 _INT, _VP]),
    "kvbm_sm_count": (_INT, []),
    "kvbm_kv_checksum": (_INT, [_VP, _VP, _VP, _VP]),
    "kvbm_rmsnorm": (_INT, [_VP, _VP, _VP, _VP, _I64, _INT, _F32, _VP]),
    "kvbm_rope_kv_write": (
        _INT,
        [_VP, _I64, _INT, _INT, _INT, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _VP],
    ),
    "kvbm_rope_kv_push": (
        _INT,
        [_VP, _I64, _INT, _INT, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _VP, _VP, _I64, _I64, _I64, _INT,
         _INT, _VP, _VP],
    ),
    "kvbm_rope_kv_push_heads": (
        _INT,
        [_VP, _I64, _INT, _INT, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _VP, _VP, _I64, _I64, _I64, _INT,
         _INT, _VP, _INT, _VP],
    ),
    "kvbm_rope_kv_write_qout": (
        _INT,
        [_VP, _I64, _INT, _INT, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _VP, _VP],
    ),
    "kvbm_rope_set_unroll": (_INT, [_INT]),
    "kvbm_silu_mul": (_INT, [_VP, _VP, _I64, _INT, _VP]),
    "kvbm_paged_decode_attn": (
        _INT,
        [_VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _INT, _VP, _INT, _INT, _INT, _INT, _F32, _INT, _VP, _VP, _VP,
         _VP],
    ),
    "kvbm_paged_decode_attn_fused": (
        _INT,
        [_VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _INT, _VP, _INT, _INT, _INT, _INT, _F32, _INT, _VP, _VP, _VP,
         _VP, _VP],
    ),
    "kvbm_paged_decode_attn_simt": (
        _INT,
        [_VP, _VP, _VP, _I64, _I64, _I64, _INT, _VP, _INT, _VP, _INT, _INT, _INT, _INT, _F32, _INT, _VP, _VP, _VP,
         _VP],
    ),
    "kvbm_skinny_gemm": (_INT, [_VP, _INT, _VP, _INT, _VP, _INT, _INT, _INT, _INT, _INT, _VP, _VP, _VP]),
    "kvbm_skinny_gemm_ctas": (_INT, []),
    "kvbm_skinny_gemm_set_pdl": (_INT, [_INT]),
    "kvbm_skinny_gemm_set_mode": (_INT, [_INT]),
    "kvbm_skinny_gemm_set_timeline": (_INT, [_VP]),
    "kvbm_skinny_gemm_status": (_INT, [_INT]),
    "kvbm_gds_status": (_INT, []),
    "kvbm_gds_open": (_INT, [C.c_char_p, _INT, C.POINTER(_VP)]),
    "kvbm_gds_open_fd": (_INT, [_INT, C.POINTER(_VP)]),
    "kvbm_gds_close": (_INT, [_VP]),
    "kvbm_gds_register_buffer": (_INT, [_VP, _U64]),
    "kvbm_gds_deregister_buffer": (_INT, [_VP]),
    "kvbm_gds_io": (_I64, [_VP, _INT, _VP, _I64, _I64, _I64]),
    "kvbm_device_alloc": (_INT, [_U64, C.POINTER(_VP)]),
    "kvbm_device_free": (_INT, [_VP]),
    "kvbm_memset_async": (_INT, [_VP, _INT, _U64, _VP]),
    "kvbm_ipc_get_handle": (_INT, [_VP, C.c_char_p]),
    "kvbm_ipc_open_handle": (_INT, [C.c_char_p, C.POINTER(_VP)]),
    "kvbm_ipc_close": (_INT, [_VP]),
    "kvbm_ipc_handle_size": (_INT, []),
    "kvbm_host_alloc_mapped": (_INT, [_U64, C.POINTER(_VP)]),
    "kvbm_host_free": (_INT, [_VP]),
    "kvbm_host_register": (_INT, [_VP, _U64]),
    "kvbm_host_unregister": (_INT, [_VP]),
    "kvbm_host_device_pointer": (_INT, [_VP, C.POINTER(_VP)]),
    "kvbm_can_access_peer": (_INT, [_INT, _INT, C.POINTER(_INT)]),
    "kvbm_enable_peer_access": (_INT, [_INT]),
    "kvbm_memcpy_async": (_INT, [_VP, _VP, _U64, _VP]),
    "kvbm_memcpy_2d_async": (_INT, [_VP, _U64, _VP, _U64, _U64, _U64, _VP]),
    "kvbm_memcpy_pairs_ce": (_INT, [_VP, _VP, _U64, _U64, _VP]),
    "kvbm_get_device": (_INT, [C.POINTER(_INT)]),
    "kvbm_error_string": (C.c_char_p, [_INT]),
}


class KvbmCudaError(RuntimeError):
    pass


# Kernels launched per successful call of each entry point. The benchmark
# reports how many of this library's kernels ran inside its timed region.
_KERNELS_PER_CALL = {
    "kvbm_kv_tile_xfer": 1, "kvbm_kv_chunk_xfer_tma": 1, "kvbm_kv_xfer": 1, "kvbm_copy_pairs": 1, "kvbm_universal_from_block": 1,
    "kvbm_block_from_universal": 1, "kvbm_nhd_hnd_transpose": 1, "kvbm_signal_flag": 1, "kvbm_wait_flag": 1,
    "kvbm_signal_flag_payload": 1, "kvbm_wait_flags_all": 1, "kvbm_rmsnorm": 1, "kvbm_rope_kv_write": 1,
    "kvbm_rope_kv_push": 1, "kvbm_rope_kv_write_qout": 1, "kvbm_rope_kv_push_heads": 1,
    "kvbm_silu_mul": 1, "kvbm_paged_decode_attn": 2, "kvbm_paged_decode_attn_fused": 1, "kvbm_paged_decode_attn_simt": 2,
    "kvbm_skinny_gemm": 1, "kvbm_kv_multicast": 1, "kvbm_signal_multicast": 1,
}
_launches = 0


def count_launches(n: int) -> None:
    global _launches
    _launches += n


def launch_count() -> int:
    return _launches


def lib_path() -> Path:
    return _build.CUDA_LIB


def load(build_if_missing: bool = True) -> C.CDLL:
    """Load (building first if needed) the kernel library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not path.exists() or _build._stale(path, _build.CUDA_SOURCES + _build.CUDA_HEADERS):
            if not build_if_missing:
                raise KvbmCudaError(f"kvbm_b200 CUDA library missing at {path}; run kvbm_b200._build")
            _build.build_cuda()
        lib = C.CDLL(str(path), mode=C.RTLD_GLOBAL)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(code: int, what: str = "") -> None:
    if code != 0:
        msg = load().kvbm_error_string(code)
        raise KvbmCudaError(f"{what}: CUDA error {code} ({msg.decode() if msg else '?'})")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
    count_launches(_KERNELS_PER_CALL.get(name, 0))
