"""Per-request block assignments: the ordered unassigned -> staged -> assigned
collections a request's blocks move through.

``ExternalBlockAssignments`` tracks block ids only (no guards): the ids a
scheduler allocated for one tier of one request, from sequence position
``offset`` on. New ids wait in the unassigned FIFO; ``stage_pending`` pairs
them, in order, with the sequence hashes of the request's next complete
blocks (checking that each hash's embedded position is the position it
lands on); ``commit_staged`` moves them to the assigned list, whose entry i
is sequence position ``offset + i``. Two such sets over the same sequence
zip into transfer plans: ``zip_assigned_pending(src, dst)`` pairs the source
tier's assigned ids with the destination tier's pending ids position by
position (an onboard or offload plan), ``zip_assigned`` pairs two assigned
sets.

``LogicalBlockAssignments`` holds the block guards themselves (the
block manager's ``MutableBlock`` -> ``CompleteBlock`` -> ``ImmutableBlock``):
``extend_blocks`` queues allocated blocks, ``stage`` completes them with the
next sequence hashes, ``register`` registers the staged ones with the
manager, ``extend_assigned`` takes blocks found by a prefix match. Dropping
the assignments (``clear``) releases every guard back to its pool.

Every mutation validates first and then commits, so a failed call leaves the
collections as they were (the blocks of a failed ``extend_*`` come back in the
exception, nothing is leaked).

Parity: crates/kvbm-logical/src/sequence/store.rs (BlockStore),
sequence/assignments/external.rs:46-396 (ExternalBlockAssignments,
zip_assigned, zip_assigned_pending), sequence/assignments/logical.rs:57-262
(LogicalBlockAssignments and its error cases).
"""

from __future__ import annotations

from collections import deque
from typing import Any, Iterable, Iterator, Sequence

from .manager import BlockManager, CompleteBlock, ImmutableBlock, MutableBlock
from .sequence import position as hash_position


class BlockSequenceError(ValueError):
    pass


class DuplicateBlockId(BlockSequenceError):
    def __init__(self, block_id: int, blocks: list | None = None):
        super().__init__(f"duplicate block_id {block_id} already present")
        self.block_id, self.blocks = block_id, blocks or []


class OrderingViolation(BlockSequenceError):
    def __init__(self, known_id: int, new_id: int, known_index: int, first_new_index: int):
        super().__init__(f"known block_id {known_id} at index {known_index} follows new block_id {new_id} "
                         f"(first new at index {first_new_index})")
        self.known_id, self.new_id = known_id, new_id
        self.known_index, self.first_new_index = known_index, first_new_index


class PositionMismatch(BlockSequenceError):
    def __init__(self, expected: int, actual: int, block_id: int):
        super().__init__(f"block {block_id}: sequence hash at position {actual}, expected {expected}")
        self.expected, self.actual, self.block_id = expected, actual, block_id


class SequenceHashMismatch(BlockSequenceError):
    def __init__(self, pos: int, expected: int, actual: int, blocks: list):
        super().__init__(f"sequence hash mismatch at position {pos}: expected {expected:#x}, got {actual:#x}")
        self.position, self.expected, self.actual, self.blocks = pos, expected, actual, blocks


class BlockStore:
    """Three ordered collections keyed by block id: unassigned (FIFO) -> staged (FIFO) -> assigned."""

    def __init__(self):
        self.assigned: list[tuple[int, Any]] = []
        self.staged: deque[tuple[int, Any]] = deque()
        self.unassigned: deque[tuple[int, Any]] = deque()
        self._ids: set[int] = set()

    def contains(self, block_id: int) -> bool:
        return block_id in self._ids

    def validate_no_duplicates(self, ids: Sequence[int]) -> int | None:
        """The first id that is already stored or repeated within ``ids``, else None."""
        seen = set()
        for i in ids:
            if i in self._ids or i in seen:
                return i
            seen.add(i)
        return None

    def insert_unassigned(self, bid: int, val: Any = None) -> None:
        self._ids.add(bid)
        self.unassigned.append((bid, val))

    def insert_staged(self, bid: int, val: Any) -> None:
        self._ids.add(bid)
        self.staged.append((bid, val))

    def insert_assigned(self, bid: int, val: Any) -> None:
        self._ids.add(bid)
        self.assigned.append((bid, val))

    def shift_unassigned(self) -> tuple[int, Any]:
        bid, v = self.unassigned.popleft()
        self._ids.discard(bid)
        return bid, v

    def shift_staged(self) -> tuple[int, Any]:
        bid, v = self.staged.popleft()
        self._ids.discard(bid)
        return bid, v

    def pop_unassigned(self) -> tuple[int, Any] | None:
        if not self.unassigned:
            return None
        bid, v = self.unassigned.pop()
        self._ids.discard(bid)
        return bid, v

    def extend_unassigned(self, bids: Sequence[int]) -> None:
        self._ids.update(bids)
        self.unassigned.extend((b, None) for b in bids)

    def stage_front(self, values: Sequence[Any]) -> None:
        """Move the first ``len(values)`` unassigned ids to staged, pairing them with ``values``
        (the ids stay in the store, so membership does not change)."""
        pop, push = self.unassigned.popleft, self.staged.append
        for v in values:
            push((pop()[0], v))

    def commit_all_staged(self) -> int:
        n = len(self.staged)
        self.assigned.extend(self.staged)
        self.staged.clear()
        return n

    def all_block_ids(self) -> list[int]:
        return [b for b, _ in self.assigned] + [b for b, _ in self.staged] + [b for b, _ in self.unassigned]

    def take(self, which: str) -> list[tuple[int, Any]]:
        col = getattr(self, which)
        out = list(col)
        col.clear()
        for b, _ in out:
            self._ids.discard(b)
        return out

    def clear(self) -> None:
        self.assigned.clear()
        self.staged.clear()
        self.unassigned.clear()
        self._ids.clear()

    def __len__(self):
        return len(self._ids)


class ExternalBlockAssignments:
    """Block ids of one tier of one sequence, from position ``offset`` on."""

    def __init__(self, offset: int = 0):
        self._s = BlockStore()
        self.offset = int(offset)
        self._order: list[int] = []   # every id in the order it arrived (assigned, staged, unassigned)

    # -------------------------------------------------------------- counts
    def contains(self, block_id: int) -> bool:
        return self._s.contains(block_id)

    def assigned_count(self) -> int:
        return len(self._s.assigned)

    def staged_count(self) -> int:
        return len(self._s.staged)

    def unassigned_count(self) -> int:
        return len(self._s.unassigned)

    def get_assigned(self, index: int) -> tuple[int, int] | None:
        return self._s.assigned[index] if 0 <= index < len(self._s.assigned) else None

    def get_staged(self, index: int) -> tuple[int, int] | None:
        return self._s.staged[index] if 0 <= index < len(self._s.staged) else None

    def assigned_iter(self) -> Iterator[tuple[int, int]]:
        return iter(list(self._s.assigned))

    def staged_iter(self) -> Iterator[tuple[int, int]]:
        return iter(list(self._s.staged))

    def unassigned_iter(self) -> Iterator[int]:
        return iter([b for b, _ in self._s.unassigned])

    def block_ids(self) -> list[int]:
        """All ids in sequence order (assigned, then staged, then pending); do not mutate."""
        return self._order

    def assigned_ids(self, start: int = 0, stop: int | None = None) -> list[int]:
        return [b for b, _ in self._s.assigned[start:stop]]

    def clear(self) -> None:
        self._s.clear()
        self._order = []

    def take_staged(self) -> list[tuple[int, int]]:
        out = self._s.take("staged")
        self._order = self._s.all_block_ids()
        return out

    # ----------------------------------------------------------- positions
    def next_position(self) -> int:
        """Sequence position the next staged id will take."""
        return self.offset + len(self._s.assigned) + len(self._s.staged)

    def assigned_positions(self) -> range:
        return range(self.offset, self.offset + len(self._s.assigned))

    def staged_positions(self) -> range:
        s = self.offset + len(self._s.assigned)
        return range(s, s + len(self._s.staged))

    def pending_positions(self) -> range:
        s = self.next_position()
        return range(s, s + len(self._s.unassigned))

    def get_at_position(self, abs_pos: int) -> tuple[int, int] | None:
        return self.get_assigned(abs_pos - self.offset) if abs_pos >= self.offset else None

    def get_pending_at_position(self, abs_pos: int) -> int | None:
        i = abs_pos - self.next_position()
        return self._s.unassigned[i][0] if 0 <= i < len(self._s.unassigned) else None

    # ------------------------------------------------------------ mutation
    def extend_block_ids(self, block_ids: Iterable[int]) -> None:
        """``block_ids`` is the full ordered list allocated to this set: ids already known must form a
        prefix (they are skipped), the rest are queued as unassigned."""
        ids = [int(b) for b in block_ids]
        known = self._s._ids
        k = 0
        while k < len(ids) and ids[k] in known:  # the known prefix is skipped
            k += 1
        new = ids[k:]
        if new and (known.intersection(new) or len(set(new)) != len(new)):
            seen = set()
            for i, bid in enumerate(new, start=k):
                if bid in known:
                    raise OrderingViolation(bid, new[0], i, k)
                if bid in seen:
                    raise DuplicateBlockId(bid)
                seen.add(bid)
        self._s.extend_unassigned(new)
        self._order.extend(new)

    def extend_assigned(self, items: Iterable[tuple[int, int]]) -> int:
        """Known ``(block_id, sequence_hash)`` pairs (cache hits) straight into the assigned list."""
        items = [(int(b), int(h)) for b, h in items]
        dup = self._s.validate_no_duplicates([b for b, _ in items])
        if dup is not None:
            raise DuplicateBlockId(dup)
        for b, h in items:
            self._s.insert_assigned(b, h)
        if self._s.staged or self._s.unassigned:
            self._order = self._s.all_block_ids()
        else:
            self._order.extend(b for b, _ in items)
        return len(items)

    def stage_pending(self, sequence_hashes: Sequence[int], limit: int | None = None) -> range:
        """Pair unassigned ids with ``sequence_hashes[next_position():limit]`` (hash i of the whole
        sequence at index i); returns the range of new staged indices."""
        st = self._s
        start_idx = len(st.staged)
        start = self.offset + len(st.assigned) + start_idx
        end = len(sequence_hashes) if limit is None else min(int(limit), len(sequence_hashes))
        if end <= start or not st.unassigned:  # the per-step common case: nothing new to pair
            return range(start_idx, start_idx)
        n = min(end - start, len(st.unassigned))
        vals = [int(h) for h in sequence_hashes[start: start + n]]
        for i, h in enumerate(vals):
            if (h >> 128) != start + i:  # a sequence hash carries its block position in its top bits
                raise PositionMismatch(start + i, hash_position(h), st.unassigned[i][0])
        st.stage_front(vals)
        return range(start_idx, start_idx + n)

    def commit_staged(self) -> range:
        start = len(self._s.assigned)
        return range(start, start + self._s.commit_all_staged())

    def assign_pending(self, sequence_hashes: Sequence[int], limit: int | None = None) -> range:
        self.stage_pending(sequence_hashes, limit)
        return self.commit_staged()


def zip_assigned(a: ExternalBlockAssignments, b: ExternalBlockAssignments) -> list[tuple[int, int, int]]:
    """``(position, a_id, b_id)`` for every position assigned in both, ascending."""
    ra, rb = a.assigned_positions(), b.assigned_positions()
    return [(p, a.get_at_position(p)[0], b.get_at_position(p)[0])
            for p in range(max(ra.start, rb.start), min(ra.stop, rb.stop))]


def zip_assigned_pending(src: ExternalBlockAssignments, dst: ExternalBlockAssignments) -> list[tuple[int, int, int]]:
    """``(position, src_id, dst_id)`` where ``src`` has the block assigned and ``dst`` a pending id for
    that position: which source block to copy into which destination block."""
    rs, rd = src.assigned_positions(), dst.pending_positions()
    return [(p, src.get_at_position(p)[0], dst.get_pending_at_position(p))
            for p in range(max(rs.start, rd.start), min(rs.stop, rd.stop))]


class LogicalBlockAssignments:
    """The block guards of one sequence in one block manager, in lifecycle order."""

    def __init__(self):
        self._s = BlockStore()

    def assigned_count(self) -> int:
        return len(self._s.assigned)

    def staged_count(self) -> int:
        return len(self._s.staged)

    def unassigned_count(self) -> int:
        return len(self._s.unassigned)

    def is_empty(self) -> bool:
        return len(self._s) == 0

    def contains(self, block_id: int) -> bool:
        return self._s.contains(block_id)

    def get_assigned(self, index: int) -> tuple[int, ImmutableBlock] | None:
        return self._s.assigned[index] if 0 <= index < len(self._s.assigned) else None

    def get_staged(self, index: int) -> tuple[int, CompleteBlock] | None:
        return self._s.staged[index] if 0 <= index < len(self._s.staged) else None

    def get_unassigned(self, index: int) -> tuple[int, MutableBlock] | None:
        return self._s.unassigned[index] if 0 <= index < len(self._s.unassigned) else None

    def assigned_iter(self):
        return iter(list(self._s.assigned))

    def staged_iter(self):
        return iter(list(self._s.staged))

    def unassigned_iter(self):
        return iter(list(self._s.unassigned))

    def all_block_ids(self) -> list[int]:
        return self._s.all_block_ids()

    def sequence_hashes(self) -> list[int]:
        return [b.sequence_hash for _, b in self._s.assigned]

    # ------------------------------------------------------------ mutation
    def extend_blocks(self, blocks: Iterable[MutableBlock]) -> int:
        blocks = list(blocks)
        dup = self._s.validate_no_duplicates([b.block_id for b in blocks])
        if dup is not None:
            raise DuplicateBlockId(dup, blocks)
        for b in blocks:
            self._s.insert_unassigned(b.block_id, b)
        return len(blocks)

    def extend_assigned(self, blocks: Iterable[ImmutableBlock], expected_hashes: Sequence[int] | None = None) -> int:
        """Matched blocks into the assigned list; with ``expected_hashes`` (the sequence's hashes from
        the next assigned position on) each block's hash is checked first."""
        blocks = list(blocks)
        dup = self._s.validate_no_duplicates([b.block_id for b in blocks])
        if dup is not None:
            raise DuplicateBlockId(dup, blocks)
        if expected_hashes is not None:
            base = len(self._s.assigned)
            for i, b in enumerate(blocks):
                if i >= len(expected_hashes) or int(expected_hashes[i]) != b.sequence_hash:
                    exp = int(expected_hashes[i]) if i < len(expected_hashes) else 0
                    raise SequenceHashMismatch(base + i, exp, b.sequence_hash, blocks)
        for b in blocks:
            self._s.insert_assigned(b.block_id, b)
        return len(blocks)

    def stage(self, sequence_hashes: Sequence[int]) -> int:
        """Complete unassigned blocks in FIFO order with the given hashes (one per block); stages
        ``min(len(sequence_hashes), unassigned)`` blocks."""
        n = min(len(sequence_hashes), len(self._s.unassigned))
        for i in range(n):
            bid, blk = self._s.shift_unassigned()
            self._s.insert_staged(bid, blk.complete(int(sequence_hashes[i])))
        return n

    def register(self, manager: BlockManager) -> int:
        """Register every staged block with ``manager``; they move to the assigned list."""
        n = len(self._s.staged)
        while self._s.staged:
            bid, blk = self._s.shift_staged()
            self._s.insert_assigned(bid, manager.register_block(blk))
        return n

    def pop_last_unassigned(self) -> tuple[int, MutableBlock] | None:
        return self._s.pop_unassigned()

    def take_assigned(self) -> list[tuple[int, ImmutableBlock]]:
        return self._s.take("assigned")

    def take_staged(self) -> list[tuple[int, CompleteBlock]]:
        return self._s.take("staged")

    def take_unassigned(self) -> list[tuple[int, MutableBlock]]:
        return self._s.take("unassigned")

    def clear(self) -> None:
        """Release every guard (mutable and staged blocks return to the reset pool, registered ones
        drop a reference)."""
        for _, b in list(self._s.assigned) + list(self._s.staged) + list(self._s.unassigned):
            b.release()
        self._s.clear()
