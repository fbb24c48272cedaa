"""In-tree build of the native parts of kvbm_b200.

Two shared objects are produced next to the sources' package:

* ``kvbm_b200/lib/libkvbm_cuda.so`` - every CUDA kernel and the CUDA memory
  plumbing, compiled by nvcc for sm_100a only (``-gencode
  arch=compute_100a,code=sm_100a``) with a static CUDA runtime and a plain C
  ABI (loaded with ctypes).
* ``kvbm_b200/_kvbm_core*.so`` - the CPU-side block manager core (block pool,
  sequence hashing, eviction policies, registry, KV events, planner, disk
  tier) in C++20 with pybind11 bindings.

Both are rebuilt only when a source is newer than the output. nvcc
cross-compiles without a GPU, so this runs on CPU-only hosts.
"""

from __future__ import annotations

import concurrent.futures as _cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
CUDA_LIB = LIB_DIR / "libkvbm_cuda.so"
BUILD_DIR = PKG.parent / "_build"

CUDA_SOURCES = [
    CSRC / "kernels" / "kv_xfer.cu",
    CSRC / "kernels" / "kv_multicast.cu",
    CSRC / "kernels" / "llama_ops.cu",
    CSRC / "kernels" / "kvbm_mem.cu",
    CSRC / "kernels" / "skinny_gemm_tc.cu",
    CSRC / "kernels" / "gds.cpp",
]
CUDA_HEADERS = [CSRC / "kernels" / "common.cuh", CSRC / "kernels" / "kvbm_kernels.h",
                CSRC / "kernels" / "decode_attn_mma.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; kvbm_b200 needs the CUDA 12.9 toolkit to build")
    return cand


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_cuda(verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a (and the cuFile host wrapper) and link libkvbm_cuda.so."""
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    jobs = []
    for src in CUDA_SOURCES:
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *CUDA_HEADERS]):
            cmd = [
                nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                "-Xptxas", "-v" if verbose else "-O3", "-I", str(CSRC / "kernels"), "-c", str(src), "-o", str(obj),
            ]
            jobs.append(cmd)
    if jobs:
        with _cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(_run, jobs))
    if _stale(CUDA_LIB, objs):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(CUDA_LIB), *map(str, objs), "-ldl"])
    return CUDA_LIB


CORE_SOURCES = sorted((CSRC / "core").glob("*.cpp")) if (CSRC / "core").exists() else []
CORE_HEADERS = sorted((CSRC / "core").glob("*.hpp")) if (CSRC / "core").exists() else []


def core_ext_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return PKG / ("_kvbm_core" + suffix)


def build_core() -> Path | None:
    """Compile the C++ block-manager core into the _kvbm_core extension."""
    srcs = sorted((CSRC / "core").glob("*.cpp"))
    hdrs = sorted((CSRC / "core").glob("*.hpp"))
    if not srcs:
        return None
    out = core_ext_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    import pybind11

    cxx = os.environ.get("CXX", "g++")
    inc = [f"-I{pybind11.get_include()}", f"-I{sysconfig.get_paths()['include']}", f"-I{CSRC / 'core'}"]
    flags = ["-O2", "-std=c++20", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wno-unused-function"]
    objs = []
    jobs = []
    for src in srcs:
        obj = BUILD_DIR / ("core_" + src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *hdrs]):
            jobs.append([cxx, *flags, *inc, "-c", str(src), "-o", str(obj)])
    if jobs:
        with _cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(_run, jobs))
    if _stale(out, objs):
        _run([cxx, "-shared", "-o", str(out), *map(str, objs), "-lpthread"])
    return out


def build_all(verbose: bool = False) -> None:
    build_core()
    build_cuda(verbose=verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built", CUDA_LIB, core_ext_path())
