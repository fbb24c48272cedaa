"""G4: the object-store tier under G2 / G3.

:class:`ObjectTier` moves whole blocks between an instance's G2 pools (one
per TP worker, fully contiguous pinned layouts) and an object store whose
keys carry the sequence hash and the worker rank, so TP ranks never read
each other's head shards:

* ``executor()`` - an offload-pipeline executor for G2 -> G4: writes the
  blocks' bytes with the store's parallel I/O and returns no registrations
  (G4 is not a block pool; presence is the store's own ``has``). With
  ``lock=True`` a block another instance is writing (conditional-create
  lock held) is skipped.
* ``stage(hashes, g2)`` - G4 -> G2 for the longest prefix of ``hashes``
  every worker's store holds: allocates G2 blocks, reads into them, and
  registers them (they become ordinary G2 hits). ``InstanceLeader`` calls it
  from ``find_matches`` after G2 and G3.

Parity: crates/kvbm-engine/src/object/mod.rs (ObjectBlockOps has / put /
get with rank-prefixed keys), object/s3/lock.rs (conditional-create lock),
tiering/offload (G2 -> G4 pipeline, object presence policies),
remote/search/g4.rs (G4 -> G2 staging on a find).
"""

from __future__ import annotations

from ..logical.manager import BlockManager, ImmutableBlock
from ..physical.layout import KvLayout
from ..utils.tracing import audit


def _host_ptr(layout: KvLayout, block_id: int) -> int:
    b = layout.backing
    host_base = getattr(b, "ptr", None)
    if host_base is None and hasattr(b, "data_ptr"):
        host_base = b.data_ptr()
    if host_base is None:
        raise ValueError("G4 needs host-resident G2 pools")
    if layout.kind != "fully_contiguous":
        raise ValueError("G4 moves whole blocks of fully contiguous G2 pools")
    return host_base + layout.layer_offsets[0] + block_id * layout.block_stride


class ObjectTier:
    """``g2_layouts``: the G2 pools of consecutive worker ranks starting at ``rank_base`` (a
    connector worker process holds one pool: its own rank's)."""

    def __init__(self, store, g2_layouts: list[KvLayout], lock: bool = False, rank_base: int = 0):
        self.store, self.layouts, self.lock, self.rank_base = store, list(g2_layouts), lock, int(rank_base)
        self.nbytes = self.layouts[0].config.bytes_per_block
        self.stats = {"put_blocks": 0, "skipped_locked": 0, "staged_blocks": 0, "get_misses": 0}

    def keys(self, seq_hash: int) -> list[str]:
        return [self.store.key(seq_hash, rank=self.rank_base + r) for r in range(len(self.layouts))]

    def contains(self, seq_hash: int) -> bool:
        return all(self.store.has(k) for k in self.keys(seq_hash))

    # ------------------------------------------------------------ G2 -> G4
    def put(self, hashes: list[int], g2_block_ids: list[int]) -> int:
        todo = []
        for h, b in zip(hashes, g2_block_ids):
            if self.lock and not all(self.store.try_lock(k) for k in self.keys(h)):
                self.stats["skipped_locked"] += 1
                continue
            todo.append((h, b))
        futs = []
        for r, lay in enumerate(self.layouts):
            keys = [self.store.key(h, rank=self.rank_base + r) for h, _ in todo]
            futs += self.store.put_blocks(keys, [_host_ptr(lay, b) for _, b in todo], self.nbytes)
        for f in futs:
            f.result()
        self.stats["put_blocks"] += len(todo)
        return len(todo)

    def executor(self):
        """Offload-pipeline executor for G2 -> G4 (items carry the G2 block id as ``src_block_id``)."""

        def run(items):
            self.put([i.seq_hash for i in items], [i.src_block_id for i in items])
            return None  # no destination pool to register in

        return run

    # ------------------------------------------------------------ G4 -> G2
    def get_into(self, hashes: list[int], g2_block_ids: list[int]) -> list[bool]:
        """Read the blocks of ``hashes`` into G2 blocks ``g2_block_ids`` (this tier's ranks); per
        block, whether every rank's object was there."""
        ok = [True] * len(hashes)
        for r, lay in enumerate(self.layouts):
            keys = [self.store.key(h, rank=self.rank_base + r) for h in hashes]
            res = self.store.get_blocks(keys, [_host_ptr(lay, b) for b in g2_block_ids], self.nbytes)
            ok = [a and b for a, b in zip(ok, res)]
        self.stats["get_misses"] += ok.count(False)
        self.stats["staged_blocks"] += ok.count(True)
        return ok

    def stage(self, hashes: list[int], g2: BlockManager) -> list[ImmutableBlock]:
        n = 0
        for h in hashes:  # longest prefix every rank holds
            if not self.contains(h):
                break
            n += 1
        if n == 0:
            return []
        got = g2.allocate_blocks_with_evictions(n)
        if got is None:
            return []
        blocks, _ = got
        ok = [True] * n
        for r, lay in enumerate(self.layouts):
            keys = [self.store.key(h, rank=self.rank_base + r) for h in hashes[:n]]
            res = self.store.get_blocks(keys, [_host_ptr(lay, b.block_id) for b in blocks], self.nbytes)
            ok = [a and b for a, b in zip(ok, res)]
        good = 0
        while good < n and ok[good]:
            good += 1
        self.stats["get_misses"] += n - good
        for b in blocks[good:]:
            b.release()
        staged = g2.register_mutable(blocks[:good], hashes[:good]) if good else []
        self.stats["staged_blocks"] += good
        audit("g4_stage", blocks=good)
        return staged
