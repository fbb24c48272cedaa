"""Remote search: cross-instance prefix reuse.

When a request's prefix is not cached locally, ask the hub's KV indexer
which other instance holds it, open a transfer session on that holder (it
pins the blocks), copy the blocks into the local G2 tier, register them and
close the session. The connector stalls the request meanwhile
(``get_num_new_matched_tokens`` answers "pending") and, once the pull has
landed, matches it like any local G2 hit.

Data path. Every G2 pool of an instance on the same node lives in a named
shared-memory file (``SharedPinnedBuffer`` / ``SharedHostBuffer``), so the
initiator maps the holder's pool read-only and copies the blocks host to
host, layout to layout, with no RPC carrying payload. Across nodes (no
shared file) the initiator reads the blocks' canonical bytes over the
messenger instead.

Holder side (:class:`RemoteHolder`) handlers on the instance messenger:

* ``kvbm.remote.open``  {initiator, hashes} -> {sid, block_ids, pools}
* ``kvbm.remote.read``  {sid, worker, first, count} -> canonical bytes
* ``kvbm.remote.close`` {sid}

Initiator side handler: ``kvbm.remote.pull_from`` {holder, hashes, session?}
(an operator's ``kvbmctl p2p pull`` / ``xfer``).

Initiator side (:class:`RemoteSearch`): ``search`` (hub query, self
filtered, decimated for long prompts), ``pull`` (session + copy + register)
and ``start`` (the same on a background thread, one future per request).

Parity: crates/kvbm-engine/src/remote/search/{discovery.rs, plan.rs,
composer.rs}, leader/remote_search.rs:107-161 (search, self filter,
pull_from), leader/control/modules/transfer.rs:364,512 (open_transfer_session,
pull_from_session), kvbm-config/src/remote_search.rs:54 (min_remote_tokens),
docs/remote-search-onboarding.md.
"""

from __future__ import annotations

import concurrent.futures as cf
import math
import os
import threading
import time
import warnings
from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch

from ..logical.manager import ImmutableBlock
from ..physical.layout import KvBlockLayout, KvLayout, LayoutConfig, LayoutDescriptor
from ..utils.tracing import audit

OPEN, READ, CLOSE = "kvbm.remote.open", "kvbm.remote.read", "kvbm.remote.close"
PULL = "kvbm.remote.pull_from"


@dataclass
class RemoteSearchConfig:
    enabled: bool = False
    min_remote_tokens: int | None = None  # None: any remote match (one block)
    max_query_hashes: int = 64            # longer prompts send a decimated query
    timeout: float = 10.0

    def min_blocks(self, block_size: int) -> int:
        if self.min_remote_tokens is None:
            return 1
        return max(1, math.ceil(self.min_remote_tokens / block_size))


def pool_export(layout: KvLayout, shareable: bool = True) -> dict:
    """Descriptor of a G2 pool another process can map (shared file) or read (messenger)."""
    d = layout.descriptor(with_ipc=False).to_dict()
    path = getattr(layout.backing, "path", None) if shareable else None
    d["extra"] = {"shm_path": path, "node": os.uname().nodename}
    return d


def _block_bytes(d: dict) -> int:
    """Bytes of one block of an exported pool (from its layout configuration)."""
    return LayoutConfig(**LayoutDescriptor.from_dict(d).config).bytes_per_block


def _map_pool(d: dict) -> KvLayout | None:
    """Map a peer's shared-file G2 pool into this process (None when not reachable)."""
    extra = d.get("extra") or {}
    path = extra.get("shm_path")
    if not path or extra.get("node") != os.uname().nodename or not os.path.exists(path):
        return None
    mm = np.memmap(path, dtype=np.uint8, mode="r", shape=(d["nbytes"],))
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)  # read-only mapping: only ever gathered from
        t = torch.from_numpy(np.asarray(mm).view(np.uint8))
    desc = LayoutDescriptor.from_dict(d)
    lay = KvLayout(LayoutConfig(**desc.config), desc.kind, KvBlockLayout(desc.block_layout), t.data_ptr(),
                   desc.layer_offsets, desc.block_stride, desc.outer_stride, desc.token_stride, desc.head_stride,
                   desc.nbytes, "pinned", None, t, desc.scales_offset)
    lay._mmap = mm  # keep the mapping alive with the layout
    return lay


class RemoteHolder:
    """Serves transfer sessions on this instance's G2 blocks."""

    def __init__(self, leader, g2_layouts: list[KvLayout], messenger, sessions=None, lease_s: float = 60.0,
                 shareable: bool = True, pool_source: Callable[[], list[dict]] | None = None):
        """``g2_layouts``: this process's G2 pools, one per worker rank; or, when the pools live in
        worker processes (a connector's scheduler), ``pool_source`` returns their exports (and the
        messenger read path, which needs the bytes here, is not offered)."""
        from ..parallel.session import SessionManager

        self.leader, self.layouts, self.messenger = leader, list(g2_layouts), messenger
        self.pool_source = pool_source
        self.sessions = sessions or SessionManager()
        self.lease_s = lease_s  # pins of a session its initiator never closes are dropped after this
        self.shareable = shareable  # False: initiators read payload over the messenger
        self._pinned: dict[str, list[ImmutableBlock]] = {}
        self._opened: dict[str, float] = {}
        self._lock = threading.Lock()
        messenger.register_handler(OPEN, self._open)
        messenger.register_handler(READ, self._read)
        messenger.register_handler(CLOSE, self._close)

    def _expire(self) -> None:
        now = time.monotonic()
        with self._lock:
            stale = [sid for sid, t in self._opened.items() if now - t > self.lease_s]
        for sid in stale:
            self._close({"sid": sid})
            audit("transfer_session_expired", session=sid)

    def _open(self, req: dict) -> dict:
        self._expire()
        hashes = [int(h) for h in req["hashes"]]
        blocks = self.leader.g2.match_blocks(hashes)
        if (req.get("tiers") or {}).get("g3", True) and getattr(self.leader, "g3", None) is not None \
                and len(self.leader.workers) and len(blocks) < len(hashes):
            # the prefix continues in G3: stage it into G2 with this leader's workers first, so the
            # session offers the whole match (the reference's synchronous find mode)
            from .leader import FindMatchesOptions, StagingMode

            for b in blocks:
                b.release()
            blocks = self.leader.find_matches(hashes, FindMatchesOptions(staging=StagingMode.FULL)).g2_blocks
        if not blocks:
            return {"sid": None, "block_ids": []}
        s = self.sessions.open(int(req["initiator"]), int(self.leader.instance_id))
        s.attach()
        with self._lock:
            self._pinned[s.session_id] = blocks
            self._opened[s.session_id] = time.monotonic()
        audit("transfer_session_opened", session=s.session_id, initiator=str(req["initiator"]), blocks=len(blocks))
        pools = self.pool_source() if self.pool_source is not None else [pool_export(l, self.shareable)
                                                                          for l in self.layouts]
        return {"sid": s.session_id, "block_ids": [b.block_id for b in blocks], "pools": pools}

    def _read(self, req: dict) -> bytes:
        if not self.layouts:
            raise RuntimeError("this holder's G2 pools live in its worker processes: map them by their files")
        with self._lock:
            blocks = self._pinned[req["sid"]]
        ids = [b.block_id for b in blocks[req["first"]: req["first"] + req["count"]]]
        data = self.layouts[req["worker"]].gather_blocks(ids).cpu().contiguous()
        return data.view(torch.uint8).numpy().tobytes()

    def _close(self, req: dict) -> dict:
        with self._lock:
            blocks = self._pinned.pop(req["sid"], [])
            self._opened.pop(req["sid"], None)
        for b in blocks:
            b.release()
        try:
            self.sessions.get(req["sid"]).close("pulled")
            self.sessions.remove(req["sid"])
        except KeyError:
            pass
        return {"ok": True, "released": len(blocks)}

    def open_sessions(self) -> int:
        with self._lock:
            return len(self._pinned)


class RemoteSearch:
    """Initiator side: find a holder through the hub, pull into local G2."""

    def __init__(self, leader, g2_layouts: list[KvLayout], messenger, hub, block_size: int,
                 config: RemoteSearchConfig | None = None,
                 copier: Callable[[list, list[int], list[int]], None] | None = None):
        """``copier(pools, src_ids, dst_ids)``, when given, moves the bytes instead of this process
        (a connector's scheduler hands the copy to its workers, whose G2 pools these are) and
        returns once they landed; ``g2_layouts`` may then be empty."""
        self.leader, self.layouts, self.messenger, self.hub = leader, list(g2_layouts), messenger, hub
        self.copier = copier
        self.block_size = block_size
        self.config = config or RemoteSearchConfig(enabled=True)
        self._pool = cf.ThreadPoolExecutor(max_workers=2, thread_name_prefix="kvbm-remote")
        self._mapped: dict[str, KvLayout] = {}
        self.stats = {"searches": 0, "hits": 0, "pulled_blocks": 0, "bytes": 0, "rpc_reads": 0}
        messenger.register_handler(PULL, self._pull_rpc)

    # -------------------------------------------------------------- search
    def _query_set(self, hashes: list[int]) -> list[int]:
        n, m = len(hashes), self.config.max_query_hashes
        if n <= m:
            return hashes
        step = math.ceil(n / (m - 1))
        picks = sorted(set(list(range(0, n, step)) + [n - 1]))
        return [hashes[i] for i in picks]

    def search(self, hashes: list[int]) -> tuple[int, int] | None:
        """(holder instance, number of leading ``hashes`` to request) or None."""
        self.stats["searches"] += 1
        if not hashes:
            return None
        d = self.hub.query(self._query_set(hashes))
        if not d.get("hit"):
            return None
        holders = [h for h in d["holders"] if h != int(self.leader.instance_id)]
        if not holders:
            return None
        pos0 = hashes[0] >> 128
        deepest = (d["hash"] >> 128) - pos0 + 1
        # a decimated query may under-report: ask for up to the next probed position
        n = min(len(hashes), deepest + math.ceil(len(hashes) / max(1, self.config.max_query_hashes - 1)))
        if n < self.config.min_blocks(self.block_size):
            return None
        return holders[0], n

    # ---------------------------------------------------------------- pull
    def pull(self, holder: int, hashes: list[int]) -> int:
        """Copy the holder's blocks for ``hashes`` (a prefix of them) into local G2; returns blocks registered.
        Opens a session on the holder (it pins the blocks), copies, and closes it."""
        addr = self.hub.peer(holder)["address"]
        resp = self.messenger.call(addr, OPEN, {"initiator": str(self.leader.instance_id),
                                                "hashes": [str(h) for h in hashes]},
                                   timeout=self.config.timeout)
        sid = resp.get("sid")
        if sid is None:
            return 0
        try:
            return self.pull_from_session(holder, resp, hashes, addr=addr)
        finally:
            self.messenger.call(addr, CLOSE, {"sid": sid}, timeout=self.config.timeout)

    def _pull_rpc(self, req: dict) -> dict:
        """``kvbm.remote.pull_from`` {holder, hashes, session?}: with ``session`` (the holder's open
        response) copy from that pinned session and leave it open, else pin + copy + unpin."""
        hashes = [int(h) for h in req["hashes"]]
        holder = int(req["holder"])
        if req.get("session"):
            n = self.pull_from_session(holder, req["session"], hashes)
        else:
            n = self.pull(holder, hashes)
        return {"pulled": n}

    def pull_from_session(self, holder: int, resp: dict, hashes: list[int], addr: str | None = None) -> int:
        """Copy the blocks of an open session (the holder's open response) into local G2 and register
        them under ``hashes``; the session stays open."""
        sid = resp.get("sid")
        if sid is None:
            return 0
        addr = addr or self.hub.peer(holder)["address"]
        audit("transfer_pull_started", session=sid, source=str(holder), blocks=len(resp["block_ids"]))
        n = len(resp["block_ids"])
        got = self.leader.g2.allocate_blocks_with_evictions(n)
        if got is None:
            return 0
        dst, _ = got
        dst_ids = [b.block_id for b in dst]
        pools = resp["pools"]
        if self.copier is not None:
            try:
                self.copier(pools, list(resp["block_ids"]), dst_ids)
            except Exception:
                for b in dst:
                    b.release()
                raise
            self.stats["bytes"] += n * _block_bytes(pools[0])
            return self._register_pulled(dst, hashes, n, sid)
        if len(pools) != len(self.layouts):
            raise ValueError(f"holder has {len(pools)} workers, this instance {len(self.layouts)}")
        for w, (pd, mine) in enumerate(zip(pools, self.layouts)):
            src = self._mapped.get(pd["extra"].get("shm_path") or "")
            if src is None:
                src = _map_pool(pd)
                if src is not None:
                    self._mapped[pd["extra"]["shm_path"]] = src
            if src is not None:
                mine.scatter_blocks(dst_ids, src.gather_blocks(resp["block_ids"]))
            else:
                raw = self.messenger.call(addr, READ, {"sid": sid, "worker": w, "first": 0, "count": n},
                                          timeout=self.config.timeout)
                self.stats["rpc_reads"] += 1
                c = mine.config
                shape = (n, c.num_layers, c.outer_dim, c.page_size, c.num_heads, c.head_dim)
                buf = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
                data = buf.view(torch.uint8 if mine.dtype in (torch.uint8, torch.float8_e4m3fn)
                                else mine.dtype).view(shape)
                mine.scatter_blocks(dst_ids, data)
            self.stats["bytes"] += n * mine.config.bytes_per_block
        return self._register_pulled(dst, hashes, n, sid)

    def _register_pulled(self, dst, hashes: list[int], n: int, sid) -> int:
        registered = self.leader.g2.register_mutable(dst, hashes[:n])
        for b in registered:
            b.release()  # now an inactive (matchable) G2 block
        self.stats["pulled_blocks"] += n
        self.stats["hits"] += 1
        audit("transfer_pull_completed", session=sid, pulled=n)
        return n

    def find_and_pull(self, hashes: list[int]) -> int:
        found = self.search(hashes)
        if found is None:
            return 0
        holder, n = found
        return self.pull(holder, hashes[:n])

    def start(self, hashes: list[int]) -> cf.Future:
        return self._pool.submit(self.find_and_pull, list(hashes))

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        self._mapped.clear()
