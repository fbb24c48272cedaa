"""Out-of-process KV host-memory service: gRPC over a Unix socket.

The service owns host-memory pools that several serving processes on a node
share: each pool is a named shared-memory file (``/dev/shm`` or a hugepage
mount) cut into fixed-size block slots; clients map the same file and
register it with CUDA themselves (``physical.memory.SharedPinnedBuffer``),
so a G2 tier can outlive, and be shared between, engine processes. The
service allocates and frees slots, keeps a hash -> slot registry so a block
written by one client can be found by another, and reports statistics.

RPCs (msgpack payloads over gRPC generic unary handlers, service
``kvbm.KvbmService``): CreatePool, Allocate, Free, Register, Lookup, Stats,
Health.

Parity: crates/kvbm-service/src/{server/grpc.rs, registry/* (registration
keys), pool/{mod,slab}.rs (per-NUMA pinned slab pools, hugepage tiers)},
proto/kvbm_service.proto, crates/kvbm-client/src/*.
"""

from __future__ import annotations

import hashlib
import mmap
import os
import threading
from collections import deque
from concurrent import futures

import grpc
import msgpack

SERVICE = "kvbm.KvbmService"
METHODS = ("CreatePool", "Allocate", "Free", "Register", "Lookup", "Stats", "Health")


class HostMemoryPool:
    """A shared-memory slab of ``num_blocks`` slots of ``block_bytes``."""

    def __init__(self, name: str, num_blocks: int, block_bytes: int, directory: str = "/dev/shm",
                 lock_pages: bool = False):
        self.name, self.num_blocks, self.block_bytes = name, num_blocks, block_bytes
        self.path = os.path.join(directory, f"kvbm_svc_{name}")
        fd = os.open(self.path, os.O_RDWR | os.O_CREAT, 0o600)
        try:
            os.ftruncate(fd, num_blocks * block_bytes)
            self.mm = mmap.mmap(fd, num_blocks * block_bytes, mmap.MAP_SHARED)
        finally:
            os.close(fd)
        self.free = deque(range(num_blocks))
        self.registry: dict[str, int] = {}
        self.owner_of: dict[int, str] = {}
        self.lock = threading.Lock()

    def close(self):
        self.mm.close()
        try:
            os.unlink(self.path)
        except FileNotFoundError:
            pass


def registration_key(name: str, num_blocks: int, block_bytes: int) -> str:
    return hashlib.sha256(f"{name}:{num_blocks}:{block_bytes}".encode()).hexdigest()[:32]


class KvbmService:
    def __init__(self, directory: str = "/dev/shm"):
        self.directory = directory
        self.pools: dict[str, HostMemoryPool] = {}
        self.lock = threading.Lock()

    # each handler takes and returns a dict
    def CreatePool(self, req):
        key = registration_key(req["name"], req["num_blocks"], req["block_bytes"])
        with self.lock:
            pool = self.pools.get(req["name"])
            if pool is None:
                pool = HostMemoryPool(req["name"], req["num_blocks"], req["block_bytes"], self.directory)
                self.pools[req["name"]] = pool
            elif (pool.num_blocks, pool.block_bytes) != (req["num_blocks"], req["block_bytes"]):
                raise ValueError("pool exists with a different geometry")
        return {"path": pool.path, "key": key, "num_blocks": pool.num_blocks, "block_bytes": pool.block_bytes}

    def _pool(self, name):
        try:
            return self.pools[name]
        except KeyError:
            raise KeyError(f"unknown pool {name!r}") from None

    def Allocate(self, req):
        p = self._pool(req["pool"])
        n = int(req["count"])
        with p.lock:
            if len(p.free) < n:
                return {"ok": False, "ids": [], "available": len(p.free)}
            ids = [p.free.popleft() for _ in range(n)]
        return {"ok": True, "ids": ids}

    def Free(self, req):
        p = self._pool(req["pool"])
        with p.lock:
            for i in req["ids"]:
                h = p.owner_of.pop(i, None)
                if h is not None:
                    p.registry.pop(h, None)
                p.free.append(i)
        return {"ok": True, "available": len(p.free)}

    def Register(self, req):
        p = self._pool(req["pool"])
        with p.lock:
            for h, i in zip(req["hashes"], req["ids"]):
                p.registry[str(h)] = int(i)
                p.owner_of[int(i)] = str(h)
        return {"ok": True}

    def Lookup(self, req):
        p = self._pool(req["pool"])
        with p.lock:
            return {"ids": [p.registry.get(str(h), -1) for h in req["hashes"]]}

    def Stats(self, req):
        with self.lock:
            return {name: {"num_blocks": p.num_blocks, "free": len(p.free), "registered": len(p.registry)}
                    for name, p in self.pools.items()}

    def Health(self, req):
        return {"status": "ok", "pools": len(self.pools)}

    def close(self):
        for p in self.pools.values():
            p.close()


def _unary(fn):
    def handler(request: bytes, context):
        try:
            out = fn(msgpack.unpackb(request, raw=False) if request else {})
            return msgpack.packb({"ok": True, "result": out}, use_bin_type=True)
        except Exception as e:  # noqa: BLE001 - returned to the client
            return msgpack.packb({"ok": False, "error": f"{type(e).__name__}: {e}"}, use_bin_type=True)
    return grpc.unary_unary_rpc_method_handler(handler, request_deserializer=None, response_serializer=None)


def serve(socket_path: str, directory: str = "/dev/shm", max_workers: int = 8):
    """Start the service on ``unix://socket_path``; returns (grpc_server, service)."""
    svc = KvbmService(directory)
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers))
    handlers = {m: _unary(getattr(svc, m)) for m in METHODS}
    server.add_generic_rpc_handlers((grpc.method_handlers_generic_handler(SERVICE, handlers),))
    server.add_insecure_port(f"unix://{socket_path}")
    server.start()
    return server, svc


def main(argv=None):
    import argparse
    import time

    p = argparse.ArgumentParser(description="kvbm host-memory service (gRPC over a Unix socket)")
    p.add_argument("--socket", default="/tmp/kvbm.sock")
    p.add_argument("--dir", default="/dev/shm")
    a = p.parse_args(argv)
    server, svc = serve(a.socket, a.dir)
    print(f"kvbm service on unix://{a.socket}", flush=True)
    try:
        while True:
            time.sleep(3600)
    except KeyboardInterrupt:
        server.stop(1)
        svc.close()


if __name__ == "__main__":
    main()
