"""Model checks of the skinny GEMM's cross-CTA protocols (csrc/kernels/skinny_gemm_tc.cu).

1. The stream-K fix-up: the schedule (whole tiles first, then equal unit ranges),
   red.add into the workspace, a ticket per tile, the last contributor converting
   the tile and re-zeroing workspace and ticket - under random completion orders
   and over repeated launches.
2. The cluster split-K handshake, below.

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


def _stream_k_launch(tiles, chunks, ctas, rng, ws, tickets, partial_of):
    """One launch of the stream-K GEMM's tile fix-up: CTAs finish their segments in a random
    order; a partial segment adds into the workspace, takes a ticket, and the tile's last
    contributor converts the sum and re-zeroes workspace and ticket. Returns the converted tiles."""
    grid = ctas
    rounds = tiles // grid
    rest = (tiles - rounds * grid) * chunks
    per = -(-rest // grid) if rest else 1
    if rounds == 0:
        grid = -(-rest // per)
    tile0 = rounds * grid
    segs = []
    for b in range(grid):
        for r in range(rounds):
            segs.append((b, r * grid + b, 0, chunks))
        u, u1 = min(b * per, (tiles - tile0) * chunks), min((b + 1) * per, (tiles - tile0) * chunks)
        while u < u1:
            t = u // chunks
            end = min(u1, (t + 1) * chunks)
            segs.append((b, tile0 + t, u - t * chunks, end - t * chunks))
            u = end
    rng.shuffle(segs)
    out = {}
    for b, tile, c0, c1 in segs:
        val = partial_of(tile, c0, c1)
        if c0 == 0 and c1 == chunks:
            assert tile not in out
            out[tile] = val                      # whole tile: stored directly
            continue
        t = tile - tile0
        first, last = (t * chunks) // per, ((t + 1) * chunks - 1) // per
        ws[tile] += val                          # red.add
        ticket = tickets[tile]
        tickets[tile] += 1
        if ticket == last - first:               # last contributor converts and re-arms
            assert tile not in out
            out[tile] = ws[tile]
            ws[tile] = 0
            tickets[tile] = 0
    return out


@pytest.mark.parametrize("tiles,chunks,ctas", [(48, 64, 148), (224, 64, 148), (32, 224, 148), (3, 7, 5), (8, 9, 11)])
def test_stream_k_fixup_converts_each_tile_once_and_rearms(tiles, chunks, ctas):
    rng = random.Random(tiles * 1000 + chunks)

    def partial_of(tile, c0, c1):  # the sum over a chunk range of a tile-specific value
        return sum((tile + 1) * (c + 1) for c in range(c0, c1))

    ws, tickets = [0] * tiles, [0] * tiles
    for launch in range(3):  # the workspace and tickets must be ready for the next launch
        out = _stream_k_launch(tiles, chunks, ctas, rng, ws, tickets, partial_of)
        assert sorted(out) == list(range(tiles))
        for tile, v in out.items():
            assert v == partial_of(tile, 0, chunks), (launch, tile)
        assert ws == [0] * tiles and tickets == [0] * tiles
