"""CPU tests of the schedule/apply sequence protocol."""

import pytest

from kvbm_b200.logical.manager import BlockManager, Tier
from kvbm_b200.logical.schedulable import DecodeOutcome, SchedulableSequence, ScheduleError, SeqState

BS = 4


def test_prefill_decode_lifecycle_and_outcomes():
    m = BlockManager(16, BS, "lru", Tier.G1)
    s = SchedulableSequence(list(range(8)), BS, max_output_tokens=6)
    s.schedule_prefill(8, m)
    assert s.state == SeqState.PREFILL_SCHEDULED and len(s.partial) == 2
    assert s.apply_prefill(100, m) == 2 and s.kv_position == 8 and s.tail_tokens() == 1
    outcomes = []
    while not s.is_complete():
        s.schedule_decode(m)
        outcomes.append(s.apply_decode(200 + s.generated, m))
    # tokens 8..13 get KV one by one: block 2 (positions 8..11) completes on the 4th decode
    assert outcomes == [DecodeOutcome.CONTINUE] * 3 + [DecodeOutcome.BLOCK_COMPLETED, DecodeOutcome.MAX_LENGTH]
    assert s.generated == 6 and len(s.registered) == 3 and s.kv_position == 13
    with pytest.raises(ScheduleError):
        s.schedule_decode(m)
    # the registered blocks are matchable by another request with the same tokens
    other = SchedulableSequence(list(s.seq.tokens[:13]) + [1], BS, 1)
    assert other.match_and_add_prefix(m) == 3
    other.release()
    s.release()
    assert m.allocate_blocks(16) is not None
    kinds = [e for e, _ in s.history]
    assert kinds[:2] == ["schedule_prefill", "apply_prefill"] and kinds[-1] == "release"


def test_chunked_prefill_revert_and_preconditions():
    m = BlockManager(8, BS, "lru", Tier.G1)
    s = SchedulableSequence(list(range(10)), BS, 2)
    with pytest.raises(ScheduleError):
        s.schedule_decode(m)  # tail is 10 tokens, not 1
    s.schedule_prefill(6, m)
    with pytest.raises(ScheduleError):
        s.schedule_prefill(2, m)  # already scheduled
    with pytest.raises(ScheduleError):
        s.apply_prefill(5, m)  # not the last chunk
    s.revert_schedule()
    assert s.state == SeqState.IDLE and s.partial == [] and m.available_blocks() == 8
    s.schedule_prefill(6, m)
    assert s.apply_prefill(None, m) == 1  # positions 0..3 complete, 4..5 partial
    s.schedule_prefill(4, m)
    assert s.apply_prefill(77, m) == 1 and s.kv_position == 10 and s.tail_tokens() == 1
    with pytest.raises(ScheduleError):
        s.schedule_prefill(1, m)  # prompt exhausted
    s.release()


def test_speculative_accepts_prefix_and_releases_rejected_blocks():
    m = BlockManager(16, BS, "lru", Tier.G1)
    s = SchedulableSequence(list(range(7)), BS, 20)
    s.schedule_prefill(7, m)
    s.apply_prefill(50, m)  # kv 7, tokens 8 (tail = token 7)
    s.schedule_speculative(5, m)  # KV for positions 7..12 -> blocks up to 4 (positions 0..15)
    assert len(s.registered) + len(s.partial) == 4
    out = s.apply_speculative([60, 61], m)  # one accepted draft + bonus: KV 7..8 valid
    assert out == DecodeOutcome.BLOCK_COMPLETED and s.kv_position == 9 and s.tail_tokens() == 1
    assert len(s.registered) == 2 and len(s.partial) == 1  # the block for 12..15 was released
    with pytest.raises(ScheduleError):
        s.apply_speculative([1], m)  # nothing scheduled
    s.schedule_speculative(0, m)
    assert s.apply_speculative([70], m) == DecodeOutcome.CONTINUE
    s.release()
    assert m.available_blocks() == 16


def test_pool_exhaustion_leaves_state_unchanged():
    m = BlockManager(2, BS, "lru", Tier.G1)
    s = SchedulableSequence(list(range(12)), BS, 1)
    with pytest.raises(ScheduleError):
        s.schedule_prefill(12, m)
    assert s.state == SeqState.IDLE and s.partial == [] and m.available_blocks() == 2
