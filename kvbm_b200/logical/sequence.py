"""Token sequences cut into blocks with positional lineage hashes.

``TokenBlockSequence`` keeps a request's tokens, the sequence hashes of its
complete blocks (computed natively: MurmurHash3-128 over the block's tokens,
chained onto the parent block's lineage with the request salt) and the
partial tail block.

Parity: the reference takes token blocks and PositionalLineageHash from the
external dynamo-tokens crate (crates/kvbm-logical/src/sequence/,
integrations/request.rs RequestSequence); the hash values differ (that
crate is not available), the structure (position, parent, salt) does not.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np

from .. import _core_native as core


def salt_hash(salt: str | int | None) -> int:
    if salt is None or salt == "":
        return 0
    if isinstance(salt, int):
        return salt & 0xFFFFFFFFFFFFFFFF
    return core.string_salt(salt)


def position(seq_hash: int) -> int:
    return seq_hash >> 128


def parent(seq_hash: int) -> int:
    return (seq_hash >> 64) & 0xFFFFFFFFFFFFFFFF


def lineage(seq_hash: int) -> int:
    return seq_hash & 0xFFFFFFFFFFFFFFFF


def sequence_hashes(tokens: Sequence[int] | np.ndarray, block_size: int, salt: str | int | None = None,
                    parent_hash: int | None = None) -> list[int]:
    return core.sequence_hashes(np.asarray(tokens, dtype=np.int32), block_size, salt_hash(salt), parent_hash)


class TokenBlockSequence:
    """Tokens of one request and the sequence hashes of its complete blocks.

    Tokens live in a buffer that grows by doubling, so appending a decode
    token costs O(1) and a block's hash is computed once, when its last token
    arrives (the per-step path of a scheduler with hundreds of sequences)."""

    def __init__(self, tokens: Sequence[int] = (), block_size: int = 16, salt: str | int | None = None):
        self.block_size = block_size
        self.salt = salt_hash(salt)
        t = np.asarray(tokens, dtype=np.int32).ravel()
        self._buf = np.empty(max(64, 2 * t.size), dtype=np.int32)
        self._buf[: t.size] = t
        self._n = int(t.size)
        self._hashes: list[int] = core.sequence_hashes(t, block_size, self.salt, None)

    @property
    def tokens(self) -> np.ndarray:
        return self._buf[: self._n]

    def __len__(self) -> int:
        return self._n

    @property
    def num_complete_blocks(self) -> int:
        return len(self._hashes)

    @property
    def sequence_hashes(self) -> list[int]:
        return list(self._hashes)

    def hashes_view(self) -> list[int]:
        """The complete blocks' hashes without a copy (callers must not modify the list)."""
        return self._hashes

    @property
    def partial_tokens(self) -> np.ndarray:
        return self._buf[len(self._hashes) * self.block_size: self._n]

    def _reserve(self, n: int) -> None:
        if n > self._buf.size:
            buf = np.empty(max(n, 2 * self._buf.size), dtype=np.int32)
            buf[: self._n] = self._buf[: self._n]
            self._buf = buf

    def append(self, tokens: Sequence[int] | int) -> list[int]:
        """Append tokens; returns the hashes of blocks completed by this call."""
        if isinstance(tokens, (list, tuple)) and len(tokens) == 1:
            tokens = tokens[0]  # a decode step's one token
        if isinstance(tokens, (int, np.integer)):
            if self._n >= self._buf.size:
                self._reserve(self._n + 1)
            self._buf[self._n] = tokens
            self._n += 1
            if (self._n - len(self._hashes) * self.block_size) < self.block_size:
                return []
        else:
            add = np.asarray(tokens, dtype=np.int32).ravel()
            self._reserve(self._n + add.size)
            self._buf[self._n: self._n + add.size] = add
            self._n += int(add.size)
        start = len(self._hashes) * self.block_size
        if self._n - start < self.block_size:
            return []
        parent_hash = self._hashes[-1] if self._hashes else None
        new = core.sequence_hashes(self._buf[start: self._n], self.block_size, self.salt, parent_hash)
        self._hashes.extend(new)
        return new

    def truncate(self, num_tokens: int) -> None:
        self._n = min(self._n, int(num_tokens))
        self._hashes = self._hashes[: self._n // self.block_size]
