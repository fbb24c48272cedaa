"""Control plane of conditional disaggregation on one node.

Two small services the decode and prefill instances share:

* a **prefill plane** carries remote-prefill dispatches from a decode
  leader to a prefill instance's engine: the request's token ids, its
  ``RemotePrefillParams`` and where its KV goes (the decode instance id,
  the destination G1 block ids, the mailbox slot and sequence number);
* a **peer directory** publishes what a prefill worker needs to write into
  a decode instance: its G1 pool descriptor (a CUDA IPC handle of the pool
  and its strides) and its mailbox descriptor.

Both come as an in-process version (prefill and decode in one process, e.g.
sharing a GPU), as a version over a key-value store (the
``torch.distributed`` TCPStore of the serving group) and as a version over
a directory on the node's shared-memory filesystem (engines started
independently, e.g. two vLLM servers); the plane also runs over the hub's
disaggregation queue and its prefill router. :func:`open_cd_services`
builds the pair from a URL. Messages are msgpack maps; token ids travel as
raw int32 bytes.

Parity: crates/kvbm-engine/src/remote/cd/wire.rs (PrefillPlane,
PrefillDispatch), leader/cd/plane.rs (enqueue on the hub CD queue),
crates/kvbm-physical/src/manager/mod.rs:119-138 (export_metadata /
import_metadata: here the pool descriptor), crates/kvbm-protocols/src/
disagg.rs:167 (RemotePrefillParams).
"""

from __future__ import annotations

import itertools
import os
import threading
import time
from collections import deque

import msgpack
import numpy as np


def encode_dispatch(request_id: str, tokens, params: dict, decode: dict, salt=None, lora=None) -> bytes:
    toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
    return msgpack.packb({"request_id": request_id, "tokens": toks.tobytes(), "params": params, "decode": decode,
                          "salt": salt, "lora": lora}, use_bin_type=True)


def decode_dispatch(raw: bytes) -> dict:
    d = msgpack.unpackb(raw, raw=False)
    d["tokens"] = np.frombuffer(d["tokens"], dtype=np.int32)
    return d


class PrefillPlane:
    """Dispatch queue of remote prefills, one queue per prefill instance."""

    def dispatch(self, target: int, raw: bytes) -> None:
        raise NotImplementedError

    def poll(self, instance: int, limit: int | None = None) -> list[dict]:
        """Dispatches for ``instance`` that have arrived (non-blocking)."""
        raise NotImplementedError

    def wait(self, instance: int, timeout_s: float, limit: int | None = None) -> list[dict]:
        """Like :meth:`poll`, but waits up to ``timeout_s`` for at least one."""
        deadline = time.monotonic() + timeout_s
        while True:
            got = self.poll(instance, limit)
            if got or time.monotonic() >= deadline:
                return got
            time.sleep(0.0005)


class LocalPrefillPlane(PrefillPlane):
    def __init__(self):
        self._q: dict[int, deque] = {}
        self._cv = threading.Condition()

    def dispatch(self, target, raw):
        with self._cv:
            self._q.setdefault(int(target), deque()).append(raw)
            self._cv.notify_all()

    def poll(self, instance, limit=None):
        out = []
        with self._cv:
            q = self._q.get(int(instance))
            while q and (limit is None or len(out) < limit):
                out.append(decode_dispatch(q.popleft()))
        return out

    def wait(self, instance, timeout_s, limit=None):
        self.wait_nonempty(instance, timeout_s)
        return self.poll(instance, limit)

    def wait_nonempty(self, instance, timeout_s) -> bool:
        """Wait up to ``timeout_s`` until a dispatch for ``instance`` is queued (does not take it)."""
        with self._cv:
            return self._cv.wait_for(lambda: bool(self._q.get(int(instance))), timeout=timeout_s)


class StorePrefillPlane(PrefillPlane):
    """Over a ``torch.distributed`` store: ``{prefix}/{target}/n`` counts the
    dispatches to ``target`` (an atomic add hands out the slot), message ``i``
    sits under ``{prefix}/{target}/{i}`` until the consumer takes it."""

    def __init__(self, store, prefix: str = "kvbm/cd/plane"):
        self.store, self.prefix = store, prefix
        self._next: dict[int, int] = {}

    def dispatch(self, target, raw):
        i = int(self.store.add(f"{self.prefix}/{int(target)}/n", 1))
        self.store.set(f"{self.prefix}/{int(target)}/{i}", raw)

    def poll(self, instance, limit=None):
        out = []
        inst = int(instance)
        while limit is None or len(out) < limit:
            i = self._next.get(inst, 1)
            key = f"{self.prefix}/{inst}/{i}"
            if not self.store.check([key]):
                break
            raw = self.store.get(key)
            self.store.delete_key(key)
            self._next[inst] = i + 1
            out.append(decode_dispatch(raw))
        return out


class HubPrefillPlane(PrefillPlane):
    """Over the hub's disaggregation queue (``/v1/disagg/enqueue`` / ``dequeue``).

    One queue for all prefill instances: whichever polls first serves the
    request, which is the hub's load-spreading policy for CD dispatches.
    """

    def __init__(self, client):
        self.client = client

    def dispatch(self, target, raw):
        self.client.cd_enqueue({"target": int(target), "payload": raw.hex()})

    def poll(self, instance, limit=None):
        out = []
        while limit is None or len(out) < limit:
            r = self.client.cd_dequeue()
            if not r:
                break
            out.append(decode_dispatch(bytes.fromhex(r["payload"])))
        return out


class HubRouterPlane(PrefillPlane):
    """Dispatch through the hub's prefill router (``/v1/prefill-router/dispatch``): the router
    picks the prefill worker (lowest net-new load, breaker tier) and calls its
    ``PrefillRouterHandler`` over the messenger. The call returns when that prefill is done, so
    it runs on a small thread pool: the decode scheduler never waits for it (completion reaches
    the decode side through the mailbox). The dispatch's ``target`` is only a hint."""

    def __init__(self, client, workers: int = 8, timeout: float = 300.0):
        import concurrent.futures as cf

        self.client, self.timeout = client, timeout
        self._pool = cf.ThreadPoolExecutor(max_workers=workers, thread_name_prefix="kvbm-cd-route")
        self.futures = []

    def dispatch(self, target, raw):
        d = decode_dispatch(raw)
        provided = int(d["decode"].get("provided_blocks", 0)) * 16
        self.futures.append(self._pool.submit(self.client.dispatch, int(d["tokens"].size), provided,
                                              {"payload": raw.hex(), "hint": int(target)}, self.timeout))

    def poll(self, instance, limit=None):
        raise RuntimeError("a hub-routed plane is consumed by PrefillRouterHandler, not polled")

    def close(self) -> None:
        self._pool.shutdown(wait=False)


class PeerDirectory:
    """Where each instance's G1 pool and mailbox can be found, per TP rank (a
    tensor-parallel instance publishes one entry per rank: its KV shard)."""

    def publish(self, instance: int, info: dict, rank: int = 0) -> None:
        raise NotImplementedError

    def lookup(self, instance: int, timeout_s: float = 60.0, rank: int = 0) -> dict:
        raise NotImplementedError


class LocalPeerDirectory(PeerDirectory):
    """In-process: ``info`` may hold the live objects (``pool_obj``, ``mailbox_obj``)."""

    def __init__(self):
        self._d: dict[tuple[int, int], dict] = {}
        self._cv = threading.Condition()

    def publish(self, instance, info, rank=0):
        with self._cv:
            self._d[(int(instance), int(rank))] = info
            self._cv.notify_all()

    def lookup(self, instance, timeout_s=60.0, rank=0):
        key = (int(instance), int(rank))
        with self._cv:
            if not self._cv.wait_for(lambda: key in self._d, timeout=timeout_s):
                raise TimeoutError(f"instance {instance} rank {rank} never published its pool")
            return self._d[key]


class StorePeerDirectory(PeerDirectory):
    def __init__(self, store, prefix: str = "kvbm/cd/peer"):
        self.store, self.prefix = store, prefix

    def publish(self, instance, info, rank=0):
        self.store.set(f"{self.prefix}/{int(instance)}/{int(rank)}", msgpack.packb(info, use_bin_type=True))

    def lookup(self, instance, timeout_s=60.0, rank=0):
        key = f"{self.prefix}/{int(instance)}/{int(rank)}"
        deadline = time.monotonic() + timeout_s
        while not self.store.check([key]):
            if time.monotonic() >= deadline:
                raise TimeoutError(f"instance {instance} never published its pool")
            time.sleep(0.005)
        return msgpack.unpackb(self.store.get(key), raw=False)


def _atomic_write(path: str, data: bytes) -> None:
    tmp = f"{path}.{os.getpid()}.{threading.get_ident()}.tmp"
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, path)


class FilePrefillPlane(PrefillPlane):
    """Over a directory shared by the node's engines (``/dev/shm`` by default).

    A dispatch is one file ``{root}/plane/{target}/{ns}-{pid}-{n}.msg``,
    written under a temporary name and renamed into place, so a consumer
    never reads a partial message. A consumer claims a message by renaming
    it (only one rename of a name succeeds) and then deletes it, so several
    pollers of one instance never serve the same dispatch twice. Messages
    are served in name order (their nanosecond timestamps)."""

    def __init__(self, root: str):
        self.root = os.path.join(root, "plane")
        self._n = itertools.count()

    def _dir(self, instance: int) -> str:
        d = os.path.join(self.root, str(int(instance)))
        os.makedirs(d, exist_ok=True)
        return d

    def dispatch(self, target, raw):
        name = f"{time.time_ns():020d}-{os.getpid()}-{next(self._n)}.msg"
        _atomic_write(os.path.join(self._dir(target), name), raw)

    def poll(self, instance, limit=None):
        d = self._dir(instance)
        out = []
        for name in sorted(n for n in os.listdir(d) if n.endswith(".msg")):
            if limit is not None and len(out) >= limit:
                break
            src = os.path.join(d, name)
            mine = f"{src}.{os.getpid()}.{threading.get_ident()}.claim"
            try:
                os.rename(src, mine)
            except FileNotFoundError:  # another poller claimed it
                continue
            with open(mine, "rb") as f:
                raw = f.read()
            os.unlink(mine)
            out.append(decode_dispatch(raw))
        return out


class FilePeerDirectory(PeerDirectory):
    """Pool and mailbox descriptors as files ``{root}/peer/{instance}_{rank}.bin``
    (msgpack, written atomically). ``info`` must be serialisable: an engine in
    another process maps the pool through the descriptor's IPC handles."""

    def __init__(self, root: str):
        self.root = os.path.join(root, "peer")
        os.makedirs(self.root, exist_ok=True)

    def _path(self, instance: int, rank: int) -> str:
        return os.path.join(self.root, f"{int(instance)}_{int(rank)}.bin")

    def publish(self, instance, info, rank=0):
        _atomic_write(self._path(instance, rank), msgpack.packb(info, use_bin_type=True))

    def withdraw(self, instance, rank=0) -> None:
        try:
            os.unlink(self._path(instance, rank))
        except FileNotFoundError:
            pass

    def lookup(self, instance, timeout_s=60.0, rank=0):
        path = self._path(instance, rank)
        deadline = time.monotonic() + timeout_s
        while not os.path.exists(path):
            if time.monotonic() >= deadline:
                raise TimeoutError(f"instance {instance} rank {rank} never published its pool")
            time.sleep(0.005)
        with open(path, "rb") as f:
            return msgpack.unpackb(f.read(), raw=False)


def open_cd_services(url: str) -> tuple[PrefillPlane, PeerDirectory]:
    """(plane, directory) for a URL: ``file:///path`` (a directory on this node) or
    ``store://host:port`` (a ``torch.distributed`` TCPStore that another process hosts)."""
    if url.startswith("file://"):
        root = url[len("file://"):]
        return FilePrefillPlane(root), FilePeerDirectory(root)
    if url.startswith("store://"):
        from datetime import timedelta

        import torch.distributed as dist

        host, _, port = url[len("store://"):].rpartition(":")
        store = dist.TCPStore(host or "127.0.0.1", int(port), is_master=False, timeout=timedelta(seconds=60))
        return StorePrefillPlane(store), StorePeerDirectory(store)
    raise ValueError(f"unknown disaggregation directory URL {url!r} (file:///path or store://host:port)")
