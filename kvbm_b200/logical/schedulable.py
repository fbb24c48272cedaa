"""A request's token sequence with a two-phase schedule/apply protocol.

:class:`SchedulableSequence` tracks one request against a
:class:`~kvbm_b200.logical.manager.BlockManager`: which tokens exist, how
many of them have their KV computed (``kv_position``), and which blocks hold
that KV. Every model step is two calls:

* ``schedule_prefill(n)`` / ``schedule_decode()`` /
  ``schedule_speculative(k)`` check the state and pre-allocate the blocks the
  step will write (so a step never fails half way for lack of blocks);
* ``apply_prefill(token)`` / ``apply_decode(token)`` /
  ``apply_speculative(tokens)`` commit it: advance ``kv_position``, register
  every block that became full (it turns immutable and matchable by other
  requests), append the generated tokens;
* ``revert_schedule()`` undoes a schedule, releasing its pre-allocated
  blocks newest first.

States: IDLE -> {PREFILL, DECODE, SPECULATIVE}_SCHEDULED -> IDLE. After a
prefill that produced a token, and after every decode, exactly one token
("the tail") has no KV yet; decode and speculative steps require that.
``match_and_add_prefix`` adopts already-cached leading blocks before the
first prefill. Each transition is appended to ``history``.

Parity: crates/kvbm-logical/src/integrations/scheduled.rs (SchedulableSequence
state machine, tail tokens, outcomes, revert), integrations/request.rs
(RequestSequence), sequence/assignments (block assignments).
"""

from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Sequence

from .manager import BlockManager, ImmutableBlock, MutableBlock
from .sequence import TokenBlockSequence


class SeqState(str, enum.Enum):
    IDLE = "idle"
    PREFILL_SCHEDULED = "prefill_scheduled"
    DECODE_SCHEDULED = "decode_scheduled"
    SPECULATIVE_SCHEDULED = "speculative_scheduled"


class DecodeOutcome(str, enum.Enum):
    CONTINUE = "continue"
    BLOCK_COMPLETED = "block_completed"
    MAX_LENGTH = "max_length"
    BLOCK_COMPLETED_AND_MAX_LENGTH = "block_completed_and_max_length"


class ScheduleError(RuntimeError):
    pass


@dataclass
class _Scheduled:
    kind: SeqState
    tokens: int                    # KV positions the step computes
    new_blocks: list[MutableBlock]  # pre-allocated by this schedule


class SchedulableSequence:
    def __init__(self, tokens: Sequence[int], block_size: int, max_output_tokens: int, salt=None):
        if max_output_tokens < 0:
            raise ValueError("max_output_tokens must be >= 0")
        self.seq = TokenBlockSequence(list(tokens), block_size, salt)
        self.block_size = block_size
        self.prompt_len = len(tokens)
        self.max_output_tokens = max_output_tokens
        self.kv_position = 0
        self.registered: list[ImmutableBlock] = []   # full blocks, in order
        self.partial: list[MutableBlock] = []         # blocks past the registered ones, in order
        self.state = SeqState.IDLE
        self._sched: _Scheduled | None = None
        self.history: list[tuple[str, dict]] = []

    # ------------------------------------------------------------ queries
    @property
    def total_tokens(self) -> int:
        return len(self.seq)

    @property
    def generated(self) -> int:
        return self.total_tokens - self.prompt_len

    def tail_tokens(self) -> int:
        return self.total_tokens - self.kv_position

    def is_complete(self) -> bool:
        return self.generated >= self.max_output_tokens

    def block_ids(self) -> list[int]:
        return [b.block_id for b in self.registered] + [b.block_id for b in self.partial]

    def _log(self, event: str, **kw) -> None:
        self.history.append((event, kw))

    def _blocks_for(self, kv_tokens: int) -> int:
        return -(-kv_tokens // self.block_size)

    def _reserve(self, kind: SeqState, tokens: int, manager: BlockManager) -> None:
        if self.state != SeqState.IDLE:
            raise ScheduleError(f"cannot schedule in state {self.state.value}")
        need = self._blocks_for(self.kv_position + tokens) - len(self.registered) - len(self.partial)
        new: list[MutableBlock] = []
        if need > 0:
            got = manager.allocate_blocks(need)
            if got is None:
                raise ScheduleError(f"{need} blocks needed, pool exhausted")
            new = list(got)
        self.partial.extend(new)
        self._sched = _Scheduled(kind, tokens, new)
        self.state = kind
        self._log(f"schedule_{kind.value.split('_')[0]}", tokens=tokens, new_blocks=len(new))

    def _commit_kv(self, tokens: int, manager: BlockManager) -> int:
        """Advance kv_position; register blocks that became full. Returns how many were registered."""
        self.kv_position += tokens
        full = self.kv_position // self.block_size
        n = full - len(self.registered)
        if n <= 0:
            return 0
        hashes = self.seq.sequence_hashes[len(self.registered): full]
        blocks, self.partial = self.partial[:n], self.partial[n:]
        self.registered.extend(manager.register_mutable(blocks, hashes))
        return n

    def _trim(self) -> None:
        """Release pre-allocated blocks the committed KV does not reach (newest first)."""
        keep = self._blocks_for(self.kv_position) - len(self.registered)
        while len(self.partial) > max(0, keep):
            self.partial.pop().release()

    # ------------------------------------------------------------ prefix
    def match_and_add_prefix(self, manager: BlockManager) -> int:
        """Adopt cached leading blocks (before any prefill); returns the number matched.

        The last prompt token is always computed, so at most
        ``(prompt_len - 1) // block_size`` blocks are taken.
        """
        if self.kv_position or self.registered or self.partial or self.state != SeqState.IDLE:
            raise ScheduleError("prefix matching only before the first prefill")
        limit = (self.prompt_len - 1) // self.block_size
        got = manager.match_blocks(self.seq.sequence_hashes[:limit])
        self.registered = list(got)
        self.kv_position = len(got) * self.block_size
        self._log("match_prefix", blocks=len(got))
        return len(got)

    # ----------------------------------------------------------- prefill
    def schedule_prefill(self, num_tokens: int, manager: BlockManager) -> None:
        remaining = self.prompt_len - self.kv_position
        if not 0 < num_tokens <= remaining:
            raise ScheduleError(f"prefill of {num_tokens} tokens with {remaining} prompt tokens left")
        self._reserve(SeqState.PREFILL_SCHEDULED, num_tokens, manager)

    def apply_prefill(self, generated_token: int | None, manager: BlockManager) -> int:
        """Commit the scheduled chunk; ``generated_token`` only after the prompt's last chunk."""
        s = self._expect(SeqState.PREFILL_SCHEDULED)
        if generated_token is not None and self.kv_position + s.tokens != self.prompt_len:
            raise ScheduleError("a token can only be generated by the prompt's last chunk")
        done = self._commit_kv(s.tokens, manager)
        if generated_token is not None:
            self.seq.append([int(generated_token)])
        self._finish("apply_prefill", registered=done)
        return done

    # ------------------------------------------------------------ decode
    def schedule_decode(self, manager: BlockManager) -> None:
        self._need_one_tail()
        if self.is_complete():
            raise ScheduleError("max_output_tokens reached")
        self._reserve(SeqState.DECODE_SCHEDULED, 1, manager)

    def apply_decode(self, token: int, manager: BlockManager) -> DecodeOutcome:
        self._expect(SeqState.DECODE_SCHEDULED)
        done = self._commit_kv(1, manager)
        self.seq.append([int(token)])
        self._finish("apply_decode", registered=done)
        return self._outcome(done)

    # ------------------------------------------------------- speculative
    def schedule_speculative(self, num_draft: int, manager: BlockManager) -> None:
        """Verify ``num_draft`` draft tokens: KV for the tail plus every draft is reserved."""
        self._need_one_tail()
        if num_draft < 0:
            raise ScheduleError("num_draft must be >= 0")
        self._reserve(SeqState.SPECULATIVE_SCHEDULED, 1 + num_draft, manager)

    def apply_speculative(self, tokens: Sequence[int], manager: BlockManager) -> DecodeOutcome:
        """``tokens`` = accepted drafts + the bonus token (at least one token).

        KV becomes valid for the old tail and the accepted drafts; the bonus
        token is the new tail. Blocks reserved for rejected drafts are
        released. Tokens past ``max_output_tokens`` are dropped.
        """
        s = self._expect(SeqState.SPECULATIVE_SCHEDULED)
        toks = [int(t) for t in tokens][: max(0, self.max_output_tokens - self.generated)]
        if not toks or len(toks) > s.tokens:
            raise ScheduleError(f"{len(toks)} tokens for a verification of {s.tokens - 1} drafts")
        done = self._commit_kv(len(toks), manager)
        self.seq.append(toks)
        self._trim()
        self._finish("apply_speculative", accepted=len(toks) - 1, registered=done)
        return self._outcome(done)

    # ------------------------------------------------------------ common
    def revert_schedule(self) -> None:
        s = self._expect(None)
        for b in reversed(s.new_blocks):
            self.partial.remove(b)
            b.release()
        self._finish("revert_schedule", released=len(s.new_blocks))

    def release(self) -> None:
        if self.state != SeqState.IDLE:
            self.revert_schedule()
        for b in reversed(self.partial):
            b.release()
        for b in reversed(self.registered):
            b.release()
        self.partial, self.registered = [], []
        self._log("release")

    def _expect(self, kind: SeqState | None) -> _Scheduled:
        if self._sched is None or (kind is not None and self.state != kind):
            raise ScheduleError(f"nothing of that kind scheduled (state {self.state.value})")
        return self._sched

    def _finish(self, event: str, **kw) -> None:
        self._sched = None
        self.state = SeqState.IDLE
        self._log(event, kv_position=self.kv_position, **kw)

    def _need_one_tail(self) -> None:
        if self.tail_tokens() != 1:
            raise ScheduleError(f"decode needs exactly one token without KV, have {self.tail_tokens()}")

    def _outcome(self, completed: int) -> DecodeOutcome:
        maxed = self.is_complete()
        if completed and maxed:
            return DecodeOutcome.BLOCK_COMPLETED_AND_MAX_LENGTH
        if completed:
            return DecodeOutcome.BLOCK_COMPLETED
        return DecodeOutcome.MAX_LENGTH if maxed else DecodeOutcome.CONTINUE
