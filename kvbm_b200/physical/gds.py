"""GPUDirect Storage for the G3 tier: whole blocks between a device pool and a
disk pool's file through cuFile, without the pinned-host bounce.

:func:`gds_available` reports whether cuFile can be used in this process (it
is loaded on first use; without the nvidia-fs driver it runs in its
compatibility mode). :class:`GdsFile` moves block runs with ``kvbm_gds_io``
on a thread pool, coalescing consecutive block ids into one call.

Parity: crates/kvbm-physical/src/transfer/capabilities.rs (allow_gds),
transfer/strategy.rs (device <-> disk direct plans); NIXL GDS / GDS_MT backends.
"""

from __future__ import annotations

import concurrent.futures as cf
import ctypes as C
import os

from ..ops import _lib

_status: int | None = None
PROBE_TIMEOUT_S = 15.0   # cuFile's driver open has been seen not to return in some containers
IO_TIMEOUT_S = 120.0     # per transfer call


def gds_status() -> int:
    """0 when cuFile is usable, else a reason code (1 no library, 2 missing symbols, 3 the
    driver open did not return within PROBE_TIMEOUT_S, >= 1000 driver error)."""
    global _status
    if _status is None:
        import threading

        box: list[int] = []
        t = threading.Thread(target=lambda: box.append(int(_lib.load().kvbm_gds_status())), daemon=True,
                             name="kvbm-gds-probe")
        t.start()
        t.join(PROBE_TIMEOUT_S)
        _status = box[0] if box else 3
    return _status


def gds_available() -> bool:
    return gds_status() == 0


def _runs(pairs: list[tuple[int, int]]) -> list[tuple[int, int, int]]:
    """(device block, file block) pairs -> runs (device block, file block, count) of consecutive ids."""
    out: list[tuple[int, int, int]] = []
    for d, f in pairs:
        if out and out[-1][0] + out[-1][2] == d and out[-1][1] + out[-1][2] == f:
            out[-1] = (out[-1][0], out[-1][1], out[-1][2] + 1)
        else:
            out.append((d, f, 1))
    return out


class GdsFile:
    """A block file opened for cuFile I/O: by ``path`` (O_DIRECT when the file system
    allows), or by an open descriptor ``fd`` (duplicated; works for unlinked files)."""

    def __init__(self, path: str | None, block_bytes: int, direct: bool = True, threads: int = 4,
                 fd: int | None = None):
        self.path, self.block_bytes = path, int(block_bytes)
        h = C.c_void_p()
        if fd is not None:
            rc = _lib.load().kvbm_gds_open_fd(int(fd), C.byref(h))
        else:
            if not path or not os.path.exists(path):
                raise FileNotFoundError(path)
            rc = _lib.load().kvbm_gds_open(path.encode(), 1 if direct else 0, C.byref(h))
        if rc != 0:
            raise OSError(f"cuFile open of {path if fd is None else f'fd {fd}'} failed ({rc})")
        self._h = h.value
        self._pool = cf.ThreadPoolExecutor(max_workers=threads, thread_name_prefix="kvbm-gds")

    def transfer(self, write: bool, dev_base: int, dev_block_stride: int, dev_ids, file_ids) -> None:
        """Move whole blocks: device block i lives at ``dev_base + i * dev_block_stride``
        (a fully contiguous pool, stride == block bytes), file block j at ``j * block_bytes``."""
        if dev_block_stride != self.block_bytes:
            raise ValueError("GDS moves whole contiguous blocks: device block stride must equal the block size")
        lib = _lib.load()

        def one(run):
            d, f, n = run
            nbytes = n * self.block_bytes
            got = lib.kvbm_gds_io(self._h, 1 if write else 0, dev_base, d * self.block_bytes, f * self.block_bytes,
                                  nbytes)
            if got != nbytes:
                raise OSError(f"cuFile {'write' if write else 'read'} of {nbytes} bytes at block {f}: {got}")

        for fut in [self._pool.submit(one, r) for r in _runs(list(zip(dev_ids, file_ids)))]:
            fut.result(timeout=IO_TIMEOUT_S)  # a cuFile call that never returns becomes an error here

    def close(self) -> None:
        if self._h:
            self._pool.shutdown(wait=False, cancel_futures=True)
            _lib.load().kvbm_gds_close(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
