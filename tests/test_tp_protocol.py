"""A CPU model of the fused GEMV + allreduce exchange protocol (csrc/w4a16.cu, tp_push / tp_finish),
run under random interleavings of the ranks' CTAs.

Per rank: an exchange buffer of two slots x world source ranks x columns, each cell a (value, tag)
pair written by one 8-byte store; a header with the launch epoch and an arrival count. A launch on
a rank starts after its previous launch finished (stream order; the epoch is read after the
programmatic-dependent-launch wait). Each CTA reads ep = epoch + 1, pushes its columns' partials
tagged with ep into slot ep & 1 of every rank's buffer, polls the cells of its own columns from
every rank until their tag is ep, adds them, and arrives; the last CTA of the launch stores ep as
the new epoch. The model checks that every read returns exactly the value the source rank pushed in
the same launch (no stale or overwritten cell) and that every launch completes (no deadlock), for
rank counts, CTA counts and launch sequences the runner uses."""

import random

import pytest


def run_protocol(world: int, ctas: int, cols_per_cta: int, launches: int, seed: int, drop_epoch_slot=False,
                 max_steps: int = 2_000_000):
    rng = random.Random(seed)
    ncols = ctas * cols_per_cta
    # cells[dst][slot][src][col] = (value, tag); tag 0 = never written (epochs start at 1)
    cells = [[[[(None, 0)] * ncols for _ in range(world)] for _ in range(2)] for _ in range(world)]
    epoch = [0] * world
    arrive = [0] * world
    done_launches = [0] * world
    results = []

    def value(src, ep, col):
        return (src, ep, col)

    def cta(r, e, c):
        """One CTA of launch e (0-based) on rank r, as a generator of atomic steps."""
        ep = epoch[r] + 1
        assert ep == e + 1
        slot = 0 if drop_epoch_slot else ep & 1
        cols = range(c * cols_per_cta, (c + 1) * cols_per_cta)
        for q in range(world):
            for col in cols:
                cells[q][slot][r][col] = (value(r, ep, col), ep)
                yield
        for q in range(world):
            for col in cols:
                while cells[r][slot][q][col][1] != ep:
                    yield
                got = cells[r][slot][q][col][0]
                if got != value(q, ep, col):
                    raise AssertionError(f"rank {r} launch {ep} read {got} for source {q} column {col}")
                results.append((r, ep, q, col))
                yield
        arrive[r] += 1
        if arrive[r] == ctas:
            arrive[r] = 0
            epoch[r] = ep

    def rank(r):
        for e in range(launches):
            running = [cta(r, e, c) for c in range(ctas)]
            while running:
                g = rng.choice(running)
                try:
                    next(g)
                except StopIteration:
                    running.remove(g)
                yield
            done_launches[r] += 1

    procs = [rank(r) for r in range(world)]
    steps = 0
    while procs:
        p = rng.choice(procs)
        try:
            next(p)
        except StopIteration:
            procs.remove(p)
        steps += 1
        if steps > max_steps:
            raise AssertionError("deadlock: " + str(done_launches))
    assert done_launches == [launches] * world
    assert len(results) == world * launches * world * ncols
    return results


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("ctas", [1, 3])
def test_two_slot_epoch_protocol(world, ctas):
    for seed in range(6):
        run_protocol(world, ctas, cols_per_cta=2, launches=6, seed=seed)


def test_one_slot_would_be_unsafe():
    """The same model with a single slot (every launch in slot 0) fails under some interleaving: a
    fast rank's next launch overwrites cells a slow rank has not read, so the slow rank waits for a
    tag that is gone (deadlock) - the second slot is what makes the protocol safe."""
    failures = 0
    for seed in range(40):
        try:
            run_protocol(2, 1, cols_per_cta=1, launches=4, seed=seed, drop_epoch_slot=True, max_steps=20_000)
        except AssertionError:
            failures += 1
    assert failures > 0
