"""Loader for the C++ block-manager core (``_kvbm_core``), building it in-tree
when the extension is missing or older than its sources."""

from __future__ import annotations

import importlib

from . import _build


def _load():
    out = _build.core_ext_path()
    srcs = sorted((_build.CSRC / "core").glob("*.[ch]pp"))
    if not out.exists() or _build._stale(out, srcs):
        _build.build_core()
    return importlib.import_module("kvbm_b200._kvbm_core")


_mod = _load()
globals().update({k: getattr(_mod, k) for k in dir(_mod) if not k.startswith("__")})
