"""The peer-memory amax exchange's protocol (h3_engine_b200/csrc/peer.cuh,
k_amax_exchange) as a host model: ranks run their exchanges under random
interleavings, each step of a rank one of the kernel's memory operations.

Checked: with the slot array's two halves alternating by epoch parity, every
rank reads every other rank's value of the same exchange, so every rank gets
the true max of every exchange and nobody waits forever.  With a single half
a fast rank's next store can replace a value a slow rank has not read yet;
the model finds such a schedule (the reason the halves alternate)."""
import random


def _run(world, values, halves, seed, max_steps=200000):
    """values[e][r]: rank r's amax in exchange e (epochs 1..E).  Returns the
    per-rank results, or None when the interleaving deadlocks (a rank waits on
    a word that will never carry its epoch)."""
    rng = random.Random(seed)
    E = len(values)
    slots = [[(0, 0.0)] * (halves * world) for _ in range(world)]    # (epoch, value)
    result = [[None] * world for _ in range(E)]

    def rank_prog(r):
        for e in range(1, E + 1):
            half = (e % halves) * world
            mine = values[e - 1][r]
            for q in range(world):                 # the warp's stores, one per lane
                slots[q][half + r] = (e, mine)
                yield
            m = mine
            for q in range(world):                 # each lane polls its word
                while slots[r][half + q][0] != e:
                    yield "wait"
                m = max(m, slots[r][half + q][1])
            result[e - 1][r] = m
            for _ in range(rng.randrange(3)):      # other work before the next exchange
                yield

    progs = {r: rank_prog(r) for r in range(world)}
    waiting = {}
    for _ in range(max_steps):
        if not progs:
            return result
        live = list(progs)
        r = rng.choice(live)
        try:
            state = next(progs[r])
        except StopIteration:
            del progs[r]
            continue
        waiting[r] = waiting.get(r, 0) + 1 if state == "wait" else 0
        if all(waiting.get(q, 0) > 50 for q in progs):
            return None
    return None


def _values(world, E, seed):
    rng = random.Random(seed)
    return [[rng.random() * 10 for _ in range(world)] for _ in range(E)]


def test_alternating_halves_give_every_rank_the_max():
    for world in (2, 3, 4, 8):
        for seed in range(40):
            vals = _values(world, 12, seed)
            res = _run(world, vals, halves=2, seed=seed)
            assert res is not None, (world, seed)
            for e, row in enumerate(res):
                assert row == [max(vals[e])] * world, (world, seed, e)


def test_a_single_half_can_lose_a_value():
    bad = 0
    for seed in range(200):
        vals = _values(2, 12, seed)
        res = _run(2, vals, halves=1, seed=seed)
        if res is None or any(row != [max(vals[e])] * 2 for e, row in enumerate(res)):
            bad += 1
    assert bad > 0
