"""A CPU model of the decode GEMV's shared-memory ring (csrc/w4a16.cu and csrc/w8a16.cu): one
producer fills `nbuf` stage buffers (full barrier: one phase per load), CW x WPC consumer warps take
the stages of each tile round-robin (warp phase p consumes stages p, p + WPC, ...), each stage is
released by CW arrivals on its empty barrier, and with WPC > 1 the consumer warps meet at a barrier
at the end of a tile. mbarrier waits are parity tests, so a wait passes on any completed phase of the
same parity: a warp that runs two ring rounds ahead of the producer would read a stale buffer.

The model runs random interleavings and checks every consumed buffer holds the stage the warp asked
for. The GEMV choosers only allow configurations with nbuf >= min(WPC, stages per CTA); the model
confirms those are safe and that breaking the rule gives stale reads."""

import random

import pytest

KW = 8  # consumer warps per CTA


def run_ring(CW: int, nbuf: int, nst: int, tiles: int, seed: int, max_steps: int = 1_000_000) -> None:
    rng = random.Random(seed)
    WPC = KW // CW
    full_done = [0] * nbuf   # completed phases of full[b]
    empty_arr = [0] * nbuf   # arrivals in the current phase of empty[b]
    empty_done = [0] * nbuf  # completed phases of empty[b]
    holds = [-1] * nbuf      # ring round whose stage the buffer holds
    met = {}                 # tile -> warps at the end-of-tile barrier

    def producer():
        for it in range(tiles * nst):
            rnd, b = divmod(it, nbuf)
            if it >= nbuf:
                while (empty_done[b] & 1) == ((rnd - 1) & 1):  # wait for the release of round rnd - 1
                    yield
            yield  # the copy is in flight
            holds[b] = rnd
            full_done[b] += 1
            yield

    def consumer(w):
        phase = w // CW
        for t in range(tiles):
            for ls in range(phase, nst, WPC):
                it = t * nst + ls
                rnd, b = divmod(it, nbuf)
                while (full_done[b] & 1) == (rnd & 1):  # parity wait for round rnd
                    yield
                if holds[b] != rnd:
                    raise AssertionError(f"warp {w} tile {t} stage {ls}: buffer {b} holds round {holds[b]}, not {rnd}")
                yield  # consume
                empty_arr[b] += 1
                if empty_arr[b] == CW:
                    empty_arr[b] = 0
                    empty_done[b] += 1
            if WPC > 1:  # partial sums meet in shared memory: all consumer warps at a barrier
                met.setdefault(t, set()).add(w)
                while len(met[t]) < KW:
                    yield

    procs = [producer()] + [consumer(w) for w in range(KW)]
    steps = 0
    while procs:
        p = rng.choice(procs)
        try:
            next(p)
        except StopIteration:
            procs.remove(p)
        steps += 1
        if steps > max_steps:
            raise AssertionError("deadlock")


def allowed(CW: int, nbuf: int, nst: int, tiles: int) -> bool:
    """The choosers' rule (stages per CTA = nst * tiles here)."""
    return nbuf >= min(KW // CW, nst * tiles)


@pytest.mark.parametrize("CW", [1, 2, 4, 8])
def test_allowed_configurations_never_read_stale_buffers(CW):
    n = 0
    for nbuf in range(2, 17):
        for nst in (1, 2, 3, 6, 7, 35):
            for tiles in (1, 2, 3):
                if not allowed(CW, nbuf, nst, tiles):
                    continue
                for seed in range(2):
                    run_ring(CW, nbuf, nst, tiles, seed)
                    n += 1
    assert n > 0


def test_shallow_ring_reads_stale_buffers():
    """8 warps on one 32-column chunk with a 2-stage ring and buffer reuse: some interleaving lets a
    warp pass its parity wait on a phase two rounds old (the configurations the choosers refuse)."""
    assert not allowed(1, 2, 35, 1)
    stale = 0
    for seed in range(20):
        try:
            run_ring(1, 2, 35, 1, seed)
        except AssertionError as e:
            assert "holds round" in str(e)
            stale += 1
    assert stale > 0
