"""Unlink cache files this process created when it is told to stop.

Non-persistent G3 pools unlink their file right after opening it (the
inode lives as long as the descriptor), so nothing is left behind on any
exit. Files that must stay reachable by path while the process runs - the
shared-memory G2 pools other instances map, a G3 file before its unlink -
are registered here instead: on SIGTERM / SIGINT / SIGHUP, and at
interpreter exit, every registered path is unlinked before the previous
handler runs (or the process exits with 128 + signum).

Parity: crates/kvbm-connector/src/connector/disk_cleanup.rs (register,
deregister, signal task unlinking G3 paths).
"""

from __future__ import annotations

import atexit
import os
import signal
import threading

_paths: set[str] = set()
_lock = threading.Lock()
_installed = False
_previous: dict[int, object] = {}
SIGNALS = (signal.SIGTERM, signal.SIGINT, signal.SIGHUP)


def cleanup() -> list[str]:
    """Unlink every registered path now; returns the paths removed."""
    with _lock:
        paths = list(_paths)
        _paths.clear()
    removed = []
    for p in paths:
        try:
            os.unlink(p)
            removed.append(p)
        except FileNotFoundError:
            pass
    return removed


def _handler(signum, frame):
    cleanup()
    prev = _previous.get(signum)
    if callable(prev):
        prev(signum, frame)
    elif prev == signal.SIG_IGN:
        return
    else:
        os._exit(128 + signum)


def _install() -> None:
    global _installed
    if _installed:
        return
    _installed = True
    atexit.register(cleanup)
    if threading.current_thread() is not threading.main_thread():
        return  # signal handlers can only be set from the main thread; atexit still covers normal exits
    for s in SIGNALS:
        try:
            _previous[s] = signal.getsignal(s)
            signal.signal(s, _handler)
        except (ValueError, OSError):
            pass


def register(path: str) -> None:
    with _lock:
        _paths.add(os.fspath(path))
    _install()


def deregister(path: str) -> None:
    with _lock:
        _paths.discard(os.fspath(path))


def registered() -> set[str]:
    with _lock:
        return set(_paths)
