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
    def __init__(self, tokens: Sequence[int] = (), block_size: int = 16, salt: str | int | None = None):
        self.block_size = block_size
        self.salt = salt_hash(salt)
        self._tokens = np.asarray(tokens, dtype=np.int32)
        self._hashes: list[int] = core.sequence_hashes(self._tokens, block_size, self.salt, None)

    @property
    def tokens(self) -> np.ndarray:
        return self._tokens

    def __len__(self) -> int:
        return int(self._tokens.size)

    @property
    def num_complete_blocks(self) -> int:
        return len(self._hashes)

    @property
    def sequence_hashes(self) -> list[int]:
        return list(self._hashes)

    @property
    def partial_tokens(self) -> np.ndarray:
        return self._tokens[len(self._hashes) * self.block_size:]

    def append(self, tokens: Sequence[int] | int) -> list[int]:
        """Append tokens; returns the hashes of blocks completed by this call."""
        add = np.atleast_1d(np.asarray(tokens, dtype=np.int32))
        self._tokens = np.concatenate([self._tokens, add])
        start = len(self._hashes) * self.block_size
        tail = self._tokens[start:]
        parent_hash = self._hashes[-1] if self._hashes else None
        new = core.sequence_hashes(tail, self.block_size, self.salt, parent_hash)
        self._hashes.extend(new)
        return new

    def truncate(self, num_tokens: int) -> None:
        self._tokens = self._tokens[:num_tokens]
        self._hashes = self._hashes[: num_tokens // self.block_size]
