"""G4 object tier: block-granular object store operations.

``ObjectBlockOps`` is the interface the offload pipelines and onboarding use
(``has`` / ``put`` / ``get`` of one block's bytes under a key derived from its
sequence hash, rank-prefixed for tensor-parallel shards), plus a
conditional-put lock so that exactly one writer uploads a block.

``FsObjectStore`` implements it over a directory (a local or network file
system standing in for an S3 bucket: a key is a file, a conditional put is an
``O_CREAT|O_EXCL`` create, a put is written to a temporary name and renamed so
readers never observe partial objects). Data moves between the pinned G2
pool and the store with one read/write per block.

Parity: crates/kvbm-engine/src/object/{mod.rs (ObjectBlockOps has/put/get,
rank-prefixed key formatters), s3/client.rs, s3/lock.rs (conditional-PUT
lock)}; docs/object.md.
"""

from __future__ import annotations

import ctypes
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor


class ObjectBlockOps:
    def key(self, seq_hash: int, rank: int = 0) -> str:
        return f"rank{rank}/{seq_hash:040x}"

    def has(self, key: str) -> bool:  # pragma: no cover - interface
        raise NotImplementedError

    def put(self, key: str, data: bytes | memoryview) -> None:  # pragma: no cover
        raise NotImplementedError

    def get(self, key: str) -> bytes | None:  # pragma: no cover
        raise NotImplementedError

    def try_lock(self, key: str, ttl_s: float = 60.0) -> bool:  # pragma: no cover
        raise NotImplementedError

    def unlock(self, key: str) -> None:  # pragma: no cover
        raise NotImplementedError


class FsObjectStore(ObjectBlockOps):
    def __init__(self, root: str, bucket: str = "kvbm", io_threads: int = 8):
        self.root = os.path.join(root, bucket)
        os.makedirs(self.root, exist_ok=True)
        self._pool = ThreadPoolExecutor(max_workers=io_threads, thread_name_prefix="kvbm-g4")
        self._lock = threading.Lock()
        self.stats = {"puts": 0, "gets": 0, "hits": 0, "misses": 0, "bytes_out": 0, "bytes_in": 0}

    def _path(self, key: str) -> str:
        p = os.path.join(self.root, key)
        os.makedirs(os.path.dirname(p), exist_ok=True)
        return p

    def has(self, key: str) -> bool:
        return os.path.exists(self._path(key))

    def put(self, key: str, data) -> None:
        p = self._path(key)
        tmp = f"{p}.tmp.{os.getpid()}.{threading.get_ident()}"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, p)
        with self._lock:
            self.stats["puts"] += 1
            self.stats["bytes_out"] += len(data)

    def get(self, key: str) -> bytes | None:
        try:
            with open(self._path(key), "rb") as f:
                data = f.read()
        except FileNotFoundError:
            with self._lock:
                self.stats["gets"] += 1
                self.stats["misses"] += 1
            return None
        with self._lock:
            self.stats["gets"] += 1
            self.stats["hits"] += 1
            self.stats["bytes_in"] += len(data)
        return data

    def try_lock(self, key: str, ttl_s: float = 60.0) -> bool:
        lp = self._path(key) + ".lock"
        try:
            fd = os.open(lp, os.O_CREAT | os.O_EXCL | os.O_WRONLY, 0o600)
        except FileExistsError:
            try:
                if time.time() - os.path.getmtime(lp) > ttl_s:  # stale lock: take it over
                    os.unlink(lp)
                    return self.try_lock(key, ttl_s)
            except FileNotFoundError:
                return self.try_lock(key, ttl_s)
            return False
        os.close(fd)
        return True

    def unlock(self, key: str) -> None:
        try:
            os.unlink(self._path(key) + ".lock")
        except FileNotFoundError:
            pass

    # ------------------------------------------------- block <-> pinned G2
    def put_blocks(self, keys: list[str], host_ptrs: list[int], nbytes: int) -> list:
        """Upload pinned-host block regions (returns futures)."""
        def one(k, p):
            self.put(k, (ctypes.c_uint8 * nbytes).from_address(p))
            self.unlock(k)
        return [self._pool.submit(one, k, p) for k, p in zip(keys, host_ptrs)]

    def get_blocks(self, keys: list[str], host_ptrs: list[int], nbytes: int) -> list[bool]:
        """Download objects into pinned-host block regions; False where missing."""
        def one(k, p):
            data = self.get(k)
            if data is None or len(data) != nbytes:
                return False
            ctypes.memmove(p, data, nbytes)
            return True
        return [f.result() for f in [self._pool.submit(one, k, p) for k, p in zip(keys, host_ptrs)]]

    def close(self) -> None:
        self._pool.shutdown(wait=True)
