"""Client of the host-memory service (``kvbm_b200.service.server``).

Parity: crates/kvbm-client/src/{client.rs, handle.rs}.
"""

from __future__ import annotations

import mmap
import os

import grpc
import msgpack

from .server import METHODS, SERVICE


class ServiceError(RuntimeError):
    pass


class KvbmServiceClient:
    def __init__(self, socket_path: str, timeout: float = 10.0):
        self.channel = grpc.insecure_channel(f"unix://{socket_path}")
        self.timeout = timeout
        self._stubs = {m: self.channel.unary_unary(f"/{SERVICE}/{m}") for m in METHODS}

    def _call(self, method: str, **req):
        raw = self._stubs[method](msgpack.packb(req, use_bin_type=True), timeout=self.timeout)
        out = msgpack.unpackb(raw, raw=False)
        if not out["ok"]:
            raise ServiceError(out["error"])
        return out["result"]

    def health(self):
        return self._call("Health")

    def create_pool(self, name: str, num_blocks: int, block_bytes: int) -> "PoolHandle":
        r = self._call("CreatePool", name=name, num_blocks=num_blocks, block_bytes=block_bytes)
        return PoolHandle(self, name, r["path"], num_blocks, block_bytes)

    def allocate(self, pool: str, count: int) -> list[int] | None:
        r = self._call("Allocate", pool=pool, count=count)
        return r["ids"] if r["ok"] else None

    def free(self, pool: str, ids: list[int]) -> int:
        return self._call("Free", pool=pool, ids=list(ids))["available"]

    def register(self, pool: str, hashes: list[int], ids: list[int]) -> None:
        self._call("Register", pool=pool, hashes=[str(h) for h in hashes], ids=list(ids))

    def lookup(self, pool: str, hashes: list[int]) -> list[int]:
        return self._call("Lookup", pool=pool, hashes=[str(h) for h in hashes])["ids"]

    def stats(self):
        return self._call("Stats")

    def close(self):
        self.channel.close()


class PoolHandle:
    """A mapped view of a service pool (register it with CUDA to use it as G2)."""

    def __init__(self, client: KvbmServiceClient, name: str, path: str, num_blocks: int, block_bytes: int):
        self.client, self.name, self.path = client, name, path
        self.num_blocks, self.block_bytes = num_blocks, block_bytes
        fd = os.open(path, os.O_RDWR)
        try:
            self.mm = mmap.mmap(fd, num_blocks * block_bytes, mmap.MAP_SHARED)
        finally:
            os.close(fd)

    def block(self, i: int) -> memoryview:
        return memoryview(self.mm)[i * self.block_bytes:(i + 1) * self.block_bytes]

    def close(self):
        self.mm.close()
