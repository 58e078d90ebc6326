"""CPU model of the fused decode step's weight ring (csrc/decode_step.cu), no GPU needed.

The producer warp of each CTA walks the step program and arms ring slot `it` (it = 0, 1, ...) for
unit after unit of this CTA's work; consumer warps compute, from the same program, the slot number
of each unit they own. This replica of both walks checks, for the benchmark models' programs:
* every armed slot is consumed exactly once, by the warp that owns its unit, and the unit the
  consumer expects there is the unit the producer loaded (same op, chunk/item, stage and half);
* under random interleavings of the producer and the 8 consumer warps with a small ring, the
  consumer-side guard (wait until the producer has armed slot `it` before the parity wait) keeps
  every wait from completing on a phase two rounds old, and nothing deadlocks; without the guard the
  same model finds stale reads, which is why the kernel has it.
"""

import random

import pytest

CWARPS = 8
ATTN_POS = 128


def ceil_div(a, b):
    return -(-a // b)


def program(n_layers, hidden, n_heads, n_kv, inter, vocab, batch, G):
    """The op list of dk_step_create: (kind, units, stages, cta0, ncta, ksplit) per op."""
    ops = []
    nxt = 0

    def place(units):
        nonlocal nxt
        ncta = min(units, G)
        cta0 = 0 if ncta == G else nxt % G
        nxt = (cta0 + ncta) % G
        return cta0, ncta

    split = 1
    while split < 4 and (hidden // 32) * (split + 1) <= G and (inter // 256) // (split + 1) >= 2:
        split += 1
    nqkv = (n_heads + 2 * n_kv) * 128
    for _ in range(n_layers):
        ops.append(("qkv", nqkv // 32, hidden // 256, *place(nqkv // 32), 1))
        ops.append(("attn", 0, 0, nxt, 0, 1))
        nxt = (nxt + batch * n_kv * 8) % G
        ops.append(("o", hidden // 32, n_heads * 128 // 256, *place(hidden // 32), 1))
        ops.append(("gate_up", inter // 32, hidden // 256, *place(inter // 32), 1))
        if split > 1:
            cta0, ncta = nxt % G, (hidden // 32) * split
            nxt = (cta0 + ncta) % G
            ops.append(("down", hidden // 32, inter // 256, cta0, ncta, split))
        else:
            ops.append(("down", hidden // 32, inter // 256, *place(hidden // 32), 1))
    ops.append(("head", vocab // 32, hidden // 64, 0, G, 1))
    return ops


def chunk_range(op, cta, G):
    """(c0, c1, st0, st1): this CTA's chunks and K stages of each (the kernel's op_work)."""
    kind, units, stages, cta0, ncta, ksplit = op
    j = (cta - cta0 + G) % G
    if j >= ncta:
        return None
    if ksplit > 1:
        c, ks = divmod(j, ksplit)
        return c, c + 1, ks * stages // ksplit, (ks + 1) * stages // ksplit
    return j * units // ncta, (j + 1) * units // ncta, 0, stages


def attn_items(op, cta, G, batch, n_kv, pos):
    S = pos // ATTN_POS + 1
    items = batch * n_kv * S
    j = (cta - op[3] + G) % G
    return list(range(j, items, G))


def test_down_is_split_on_the_benchmark_model():
    ops = program(batch=1, G=148, **QWEN15)
    down = [op for op in ops if op[0] == "down"][0]
    assert down[5] == 3 and down[4] == 144
    small = [op for op in program(batch=1, G=148, **SMALL) if op[0] == "down"][0]
    assert small[5] == 2  # the test model exercises the split path too


def producer_walk(ops, cta, G, batch, n_kv, pos):
    """The unit loaded into each slot, in arming order."""
    seq = []
    for j, op in enumerate(ops):
        kind, units, stages = op[:3]
        if kind == "attn":
            for item in attn_items(op, cta, G, batch, n_kv, pos):
                for blk in range(8):
                    for kv in range(2):
                        seq.append((j, item, blk, kv))
            continue
        r = chunk_range(op, cta, G)
        if r is None:
            continue
        c0, c1, st0, st1 = r
        if kind == "head":
            nch = c1 - c0
            for rnd in range(ceil_div(nch, 8)):
                nr = min(8, nch - 8 * rnd)
                for k in range(stages):
                    for w in range(nr):
                        seq.append((j, c0 + 8 * rnd + w, k, 0))
            continue
        halves = 2 if kind == "gate_up" else 1
        nst = st1 - st0
        for u in range((c1 - c0) * nst):
            for h in range(halves):
                seq.append((j, c0 + u // nst, st0 + u % nst, h))
    return seq


def consumer_walk(ops, cta, G, batch, n_kv, pos, warp):
    """(slot number, unit) of each unit warp `warp` consumes, in its order (the kernel's run_int4,
    run_head and run_attention_item indexing)."""
    out = []
    base = 0
    for j, op in enumerate(ops):
        kind, units, stages = op[:3]
        if kind == "attn":
            b = base
            for item in attn_items(op, cta, G, batch, n_kv, pos):
                out.append((b + 2 * warp, (j, item, warp, 0)))
                out.append((b + 2 * warp + 1, (j, item, warp, 1)))
                b += 16
            base = b
            continue
        r = chunk_range(op, cta, G)
        if r is None:
            continue
        c0, c1, st0, st1 = r
        if kind == "head":
            nch = c1 - c0
            rbase = base
            for rnd in range(ceil_div(nch, 8)):
                nr = min(8, nch - 8 * rnd)
                if warp < nr:
                    for k in range(stages):
                        out.append((rbase + k * nr + warp, (j, c0 + 8 * rnd + warp, k, 0)))
                rbase += nr * stages
            base += nch * stages
            continue
        halves = 2 if kind == "gate_up" else 1
        nst = st1 - st0
        nunits = (c1 - c0) * nst
        for b in range(warp, nunits * halves, CWARPS):  # boxes dealt to the warps one by one
            u, h = divmod(b, halves)
            out.append((base + b, (j, c0 + u // nst, st0 + u % nst, h)))
        base += nunits * halves
    return out


QWEN15 = dict(n_layers=28, hidden=1536, n_heads=12, n_kv=2, inter=8960, vocab=151936)
SMALL = dict(n_layers=2, hidden=512, n_heads=4, n_kv=2, inter=1280, vocab=4096)


@pytest.mark.parametrize("arch", [QWEN15, SMALL])
@pytest.mark.parametrize("batch,pos", [(1, 0), (1, 767), (2, 300), (4, 1023)])
def test_consumers_find_the_producers_units(arch, batch, pos):
    G = 148
    ops = program(batch=batch, G=G, **arch)
    for cta in (0, 1, 47, 64, 100, 147):
        seq = producer_walk(ops, cta, G, batch, arch["n_kv"], pos)
        seen = {}
        for w in range(CWARPS):
            for it, unit in consumer_walk(ops, cta, G, batch, arch["n_kv"], pos, w):
                assert it not in seen, (cta, it)
                seen[it] = w
                assert seq[it] == unit, (cta, w, it, seq[it], unit)
        assert sorted(seen) == list(range(len(seq))), cta


class Deadlock(Exception):
    pass


def simulate(seqs_by_warp, n_slots, nslots, guard, rng):
    """Random interleaving of one producer and the consumer warps; returns how many waits passed on a
    stale phase. The producer arms slot numbers in order (round it // nslots of ring slot it % nslots)
    once that ring slot's previous round was released; arming and the copies landing are merged into
    one step (the barrier's completed-phase count c goes up). A consumer waits for round r of its slot
    with try_wait.parity(r & 1), which passes whenever c % 2 != r % 2 - correct if c == r + 1, stale if
    c <= r - 1 (the phase of round r - 2). With the guard it first waits for `issued > it`."""
    completed = [0] * nslots
    released = [0] * nslots
    issued = 0
    pc = [0] * len(seqs_by_warp)
    stale = steps = 0
    while issued < n_slots or any(pc[w] < len(q) for w, q in enumerate(seqs_by_warp)):
        steps += 1
        if steps > 100 * (n_slots + 10):
            raise Deadlock
        actors = []
        if issued < n_slots and released[issued % nslots] >= issued // nslots:
            actors.append("p")
        for w, q in enumerate(seqs_by_warp):
            if pc[w] == len(q):
                continue
            it = q[pc[w]]
            if guard and issued <= it:
                continue
            if completed[it % nslots] % 2 != (it // nslots) % 2:
                actors.append(w)
        if not actors:
            continue
        a = rng.choice(actors)
        if a == "p":
            completed[issued % nslots] += 1
            issued += 1
        else:
            it = seqs_by_warp[a][pc[a]]
            if completed[it % nslots] < it // nslots + 1:
                stale += 1
            released[it % nslots] += 1
            pc[a] += 1
    return stale


@pytest.mark.parametrize("pos", [100, 900])
def test_ring_guard_prevents_stale_phases(pos):
    G, batch = 148, 1
    ops = program(batch=batch, G=G, **QWEN15)
    rng = random.Random(1)
    for cta in (0, 64, 147):
        per_warp = [[it for it, _ in consumer_walk(ops, cta, G, batch, 2, pos, w)] for w in range(CWARPS)]
        n = len(producer_walk(ops, cta, G, batch, 2, pos))
        # the op program alone: a quarter of the layers keeps the simulation short
        cut = n // 4
        trimmed = [[it for it in s if it < cut] for s in per_warp]
        for _ in range(3):
            assert simulate(trimmed, cut, nslots=12, guard=True, rng=rng) == 0


def test_ring_without_guard_can_pass_on_an_old_phase():
    """A warp whose next slot is more than one ring round ahead of the producer passes its parity
    wait on the slot's phase of two rounds earlier without the guard (and the ring's bookkeeping then
    falls apart); with the guard every interleaving completes with no stale pass."""
    # warp 0 owns slots 0 and 9 of a 4-slot ring; warp 1 owns every other slot
    seqs = [[0, 9], [1, 2, 3, 4, 5, 6, 7, 8]]
    broken = 0
    for seed in range(50):
        try:
            broken += simulate(seqs, 10, nslots=4, guard=False, rng=random.Random(seed)) > 0
        except Deadlock:
            broken += 1
    assert broken > 0
    assert sum(simulate(seqs, 10, nslots=4, guard=True, rng=random.Random(s)) for s in range(50)) == 0
