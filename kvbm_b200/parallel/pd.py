"""Completion words of prefill -> decode transfers on one node.

The decode instance owns a :class:`HostMailbox`: one 64-bit word per
in-flight remote prefill, in page-locked host memory that every GPU of the
node can store to. A prefill worker, after pushing a request's KV into the
decode instance's G1 pool over NVLink (``ops.kv_ops.kv_transfer`` into the
pool mapped through CUDA IPC), launches a one-thread kernel behind the last
push that release-stores the request's sequence number into its word at
system scope (:class:`MailboxWriter` gives it the word's device address).
The decode worker reads the word with a plain host load from
``get_finished``; no NCCL/NIXL call and no device wait sits on the data
path.

Parity: replaces the reference's pull of prefill G2 blocks over NIXL
(crates/kvbm-engine/src/leader/instance.rs:1394 rdma_pull_with_opts ->
plan_pull G2->G2) followed by a G2->G1 onboard, and the velo event that
signals the pull's completion.
"""

from __future__ import annotations


# ---------------------------------------------------------------------------
# Host-visible mailboxes: completion of a remote prefill as the connector
# sees it (the decode worker polls host memory from ``get_finished``; no
# device wait, no host round trip through its GPU).
# ---------------------------------------------------------------------------


class HostMailbox:
    """Decode side: one u64 completion word per in-flight remote prefill.

    The words live in page-locked host memory that every GPU of the node can
    store to. A prefill GPU publishes a request by a system-scope release
    store of the request's sequence number into its slot, after the stores of
    the request's KV into this instance's pool; this process reads the word
    with a plain load, so ``get_finished`` costs no GPU work. With ``name``
    the memory is a named shared-memory file (other processes map it by
    name); without, it is private pinned memory (prefill in this process).

    Sequence numbers only grow, so a slot can be reused as soon as its
    request is reported: a stale value can never equal a newer number.

    With tensor parallelism several prefill ranks fill one decode rank's
    shard: each slot has ``words`` words, one per contributing prefill rank,
    and the request has landed once all of them read its sequence number.
    """

    def __init__(self, slots: int, name: str | None = None, words: int = 8):
        import ctypes as C
        from collections import deque

        import numpy as np

        from ..physical.memory import PinnedBuffer, SharedPinnedBuffer

        self.slots, self.name, self.words = int(slots), name, int(words)
        self.nbytes = max(4096, (self.slots * self.words * 8 + 4095) // 4096 * 4096)
        self.buf = SharedPinnedBuffer(name, self.nbytes) if name else PinnedBuffer(self.nbytes)
        arr = (C.c_uint8 * self.nbytes).from_address(self.buf.ptr)
        self._words = np.frombuffer(arr, dtype=np.uint64, count=self.slots * self.words)
        self._words[:] = 0
        self._free = deque(range(self.slots))

    def descriptor(self) -> dict:
        return {"name": self.name, "nbytes": self.nbytes, "slots": self.slots, "words": self.words}

    def alloc(self) -> int | None:
        return self._free.popleft() if self._free else None

    def free(self, slot: int) -> None:
        self._free.append(int(slot))

    @property
    def num_free(self) -> int:
        return len(self._free)

    def value(self, slot: int, contributor: int = 0) -> int:
        return int(self._words[slot * self.words + contributor])

    def landed(self, slot: int, seq: int, contributors: int = 1) -> bool:
        base = slot * self.words
        return all(int(self._words[base + c]) == seq for c in range(contributors))

    def device_ptr(self, slot: int = 0, contributor: int = 0) -> int:
        return self.buf.device_ptr + 8 * (int(slot) * self.words + int(contributor))

    def close(self) -> None:
        self._words = None
        self.buf.close()


class MailboxWriter:
    """Prefill side: the device address of another instance's mailbox words."""

    def __init__(self, desc: dict, local: HostMailbox | None = None):
        from ..physical.memory import SharedPinnedBuffer

        self.slots = int(desc["slots"])
        self.words = int(desc.get("words", 1))
        self._buf = None
        if local is not None:
            self._base = local.buf.device_ptr
        else:
            if not desc.get("name"):
                raise ValueError("a mailbox in another process must be a named shared-memory mailbox")
            self._buf = SharedPinnedBuffer(desc["name"], int(desc["nbytes"]), create=False)
            self._base = self._buf.device_ptr

    def flag_ptr(self, slot: int, contributor: int = 0) -> int:
        if not 0 <= slot < self.slots or not 0 <= contributor < self.words:
            raise IndexError(f"mailbox word ({slot}, {contributor}) out of range ({self.slots}, {self.words})")
        return self._base + 8 * (int(slot) * self.words + int(contributor))

    def close(self) -> None:
        if self._buf is not None:
            self._buf.close()
            self._buf = None
