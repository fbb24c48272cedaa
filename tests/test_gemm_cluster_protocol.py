"""Model check of the cluster split-K GEMM's shared-memory handshake.

``skinny_gemm_cluster_kernel`` (csrc/kernels/skinny_gemm_tc.cu) has S CTAs of a
cluster walk the same tiles. Per tile each CTA writes its fp32 partial into its
own shared memory, arrives on every rank's ``red_ready``, waits for its own
``red_ready``, reads its slice of every rank's partial over distributed shared
memory, and arrives on every rank's ``red_done``; it overwrites its partial
(next tile) or exits only after its own ``red_done`` phase completed. Each
mbarrier expects S arrivals per phase.

This test runs that protocol as a state machine under many random schedules
and checks what the hardware would not: that no arrival lands in a phase other
than the one its sender means (an mbarrier counts arrivals into its current
phase), that every read sees the partial of the tile being reduced, and that no
rank reads the shared memory of a rank that has left.
"""

import random

import pytest


class _Bar:
    def __init__(self, count):
        self.count, self.phase, self.pending = count, 0, count

    def arrive(self, meant_phase):
        assert meant_phase == self.phase, f"arrival for phase {meant_phase} counted in phase {self.phase}"
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, phase):
        return self.phase > phase


def _run(S, T, seed, wait_before_overwrite=True):
    rng = random.Random(seed)
    ready = [_Bar(S) for _ in range(S)]
    done = [_Bar(S) for _ in range(S)]
    partial = [None] * S
    exited = [False] * S

    def rank(r):
        for j in range(T):
            if j > 0 and wait_before_overwrite:
                while not done[r].done(j - 1):
                    yield
            partial[r] = j                 # overwrite own partial
            for q in range(S):
                ready[q].arrive(j)
                yield
            while not ready[r].done(j):
                yield
            for q in range(S):             # read every rank's partial of tile j
                assert not exited[q], f"rank {r} read rank {q} after it left"
                assert partial[q] == j, f"rank {r} saw tile {partial[q]} in rank {q}, wanted {j}"
                yield
            for q in range(S):
                done[q].arrive(j)
                yield
        while not done[r].done(T - 1):     # nobody reads this partial any more
            yield
        exited[r] = True

    procs = {r: rank(r) for r in range(S)}
    steps = 0
    while procs:
        r = rng.choice(list(procs))
        try:
            next(procs[r])
        except StopIteration:
            del procs[r]
        steps += 1
        assert steps < 100000, "no progress"
    assert all(exited)


def test_model_catches_an_early_overwrite():
    # without the red_done wait before a rank reuses its partial, some schedule must fail
    failures = 0
    for seed in range(100):
        try:
            _run(3, 3, seed, wait_before_overwrite=False)
        except AssertionError:
            failures += 1
    assert failures > 0


@pytest.mark.parametrize("S", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("T", [1, 2, 5])
def test_cluster_handshake_is_safe_under_random_schedules(S, T):
    for seed in range(60):
        _run(S, T, seed)
