"""Resume for a persistent G3 tier: a journal of which block holds which hash.

A persistent disk pool (``DiskLayout(..., persistent=True)``) keeps its file
across restarts, but the block manager's registrations live in memory. The
journal records them next to the file: before an offload writes into block
ids it logs an *invalidate* for them (their old contents are about to be
overwritten), and after the write completes it logs a *commit* of
``(block id, sequence hash)``. Replaying the journal gives the blocks whose
data is complete; :func:`restore` re-registers them in a fresh manager, so
a restarted instance finds its G3 prefix cache again. ``compact`` rewrites
the journal to one commit per live block.

Records are msgpack maps appended to one file; a torn tail (a crash in the
middle of an append) is ignored on replay.

Parity: the reference keeps no G3 index across restarts (its G3 files are
unlinked right after registration); this is the optional resume the G3
tier design allows for ("re-registration of G3 hashes").
"""

from __future__ import annotations

import os
import threading

import msgpack

from ..logical.manager import BlockManager


class TierJournal:
    def __init__(self, path: str, fsync: bool = False):
        self.path, self.fsync = path, fsync
        self._f = open(path, "ab")
        self._lock = threading.Lock()

    def _append(self, rec: dict) -> None:
        with self._lock:
            self._f.write(msgpack.packb(rec, use_bin_type=True))
            self._f.flush()
            if self.fsync:
                os.fsync(self._f.fileno())

    def invalidate(self, block_ids: list[int]) -> None:
        if block_ids:
            self._append({"op": "x", "ids": [int(i) for i in block_ids]})

    def commit(self, block_ids: list[int], hashes: list[int]) -> None:
        if block_ids:
            self._append({"op": "c", "ids": [int(i) for i in block_ids], "h": [str(h) for h in hashes]})

    @staticmethod
    def replay(path: str) -> dict[int, int]:
        """block id -> sequence hash of every block whose last record is a commit."""
        live: dict[int, int] = {}
        if not os.path.exists(path):
            return live
        with open(path, "rb") as f:
            up = msgpack.Unpacker(f, raw=False)
            try:
                for rec in up:
                    if rec.get("op") == "x":
                        for i in rec["ids"]:
                            live.pop(int(i), None)
                    elif rec.get("op") == "c":
                        for i, h in zip(rec["ids"], rec["h"]):
                            live[int(i)] = int(h)
            except (msgpack.ExtraData, msgpack.FormatError, ValueError):
                pass  # torn tail
        return live

    def compact(self, live: dict[int, int] | None = None) -> None:
        live = self.replay(self.path) if live is None else live
        tmp = self.path + ".tmp"
        with open(tmp, "wb") as f:
            ids = sorted(live)
            f.write(msgpack.packb({"op": "c", "ids": ids, "h": [str(live[i]) for i in ids]}, use_bin_type=True))
            f.flush()
            os.fsync(f.fileno())
        with self._lock:
            self._f.close()
            os.replace(tmp, self.path)
            self._f = open(self.path, "ab")

    def close(self) -> None:
        with self._lock:
            self._f.close()


def restore(manager: BlockManager, live: dict[int, int]) -> int:
    """Re-register journaled blocks in a freshly created ``manager``; returns how many.

    A fresh pool hands out every block id in ascending order, so taking all
    of them claims exactly the journaled ids; the others go straight back to
    the free list.
    """
    if not live:
        return 0
    n = manager.total_blocks()
    blocks = manager.allocate_blocks(n)
    if blocks is None or [b.block_id for b in blocks] != list(range(n)):
        raise RuntimeError("restore needs a fresh, empty pool")
    keep = [b for b in blocks if b.block_id in live]
    for b in blocks:
        if b.block_id not in live:
            b.release()
    imm = manager.register_mutable(keep, [live[b.block_id] for b in keep])
    for b in imm:
        b.release()  # cached (inactive) until matched
    return len(keep)
