"""Model check of the cross-rank protocol of the data-parallel averaging
kernel (``nano_megatron_b200/csrc/dp_reduce.cu``), on the CPU.

Each rank alternates a backward (which writes this step's gradients into its
own span) and one averaging call (new epoch) on one stream. A call is a grid
of CTAs, dispatched in block order into the SM slots that other kernels leave
free (down to one). Each CTA does what the kernel does:

1. announce ``ready[r] = e`` on every peer, wait until every peer announced e;
2. sum its part of slice r over every rank's buffer, scale, store the result
   into every rank's buffer;
3. add 1 to ``done[r]`` on every peer and to its own ``finished``; the last CTA
   of the rank waits until ``done[p]`` reached the grid size for every peer,
   then resets the counters.

Checks: every call finishes; every value read for a sum is that rank's
gradient of the current step (never a stale or a next-step value); every
rank's span holds the current step's average when its call ends; no counter
ever exceeds the grid size (no increment of the next call reaches a counter
before this call reset it). A variant without the ready wait is caught.
"""

import random
import sys

import pytest


def wait_until(cond):
    while not cond():
        yield


def wait_ready(rank, e, world):
    """Step 1's wait: every peer announced epoch ``e`` here."""
    yield from wait_until(lambda: all(rank.ready[p] >= e for p in range(world) if p != rank.r))


class Rank:
    def __init__(self, r, world, grid):
        self.r = r
        self.ready = [0] * world
        self.done = [0] * world
        self.finished = 0
        # buf[slice][part] = ("grad", step, rank) before averaging, ("avg", step) after
        self.buf = [[("unwritten",)] * grid for _ in range(world)]


def cta(rank, ranks, e, b, grid, world):
    r = rank.r

    def run():
        for p in range(world):
            if p != r:
                ranks[p].ready[r] = max(ranks[p].ready[r], e)
        yield from wait_ready(rank, e, world)
        # part b of slice r: read every rank's value, then write the average everywhere
        for p in range(world):
            v = ranks[p].buf[r][b]
            assert v == ("grad", e, p), f"rank {r} step {e}: read {v} from rank {p}"
            yield
        for p in range(world):
            ranks[p].buf[r][b] = ("avg", e)
            yield
        for p in range(world):
            if p != r:
                ranks[p].done[r] += 1
                assert ranks[p].done[r] <= grid, "an increment reached a counter before its reset"
        rank.finished += 1
        assert rank.finished <= grid
        if rank.finished == grid:
            yield from wait_until(lambda: all(rank.done[p] == grid for p in range(world) if p != r))
            rank.done = [0] * world
            rank.finished = 0
    return run()


def simulate(seed, world, steps, grid, max_slots):
    rng = random.Random(seed)
    ranks = [Rank(r, world, grid) for r in range(world)]
    st = [{"step": 1, "phase": "backward", "left": rng.randint(1, 20), "next": 0, "resident": [], "held": 0}
          for _ in range(world)]
    for _ in range(300000):
        if all(s["step"] > steps for s in st):
            return
        r = rng.randrange(world)
        s, rank = st[r], ranks[r]
        if s["step"] > steps:
            continue
        if s["phase"] == "backward":
            s["left"] -= 1
            if s["left"] <= 0:  # this step's gradients are final in the own span
                rank.buf = [[("grad", s["step"], r)] * grid for _ in range(world)]
                s["phase"], s["next"] = "reduce", 0
            continue
        if rng.random() < 0.05:
            s["held"] = rng.randint(0, max_slots - 1)
        while s["next"] < grid and len(s["resident"]) < max_slots - s["held"]:
            s["resident"].append(cta(rank, ranks, s["step"], s["next"], grid, world))
            s["next"] += 1
        if s["resident"]:
            c = rng.choice(s["resident"])
            try:
                next(c)
            except StopIteration:
                s["resident"].remove(c)
        if not s["resident"] and s["next"] == grid:
            assert all(v == ("avg", s["step"]) for row in rank.buf for v in row), \
                f"rank {r} step {s['step']}: span not fully averaged"
            s["step"] += 1
            s["phase"], s["left"] = "backward", rng.randint(1, 20)
    raise AssertionError(f"stuck: {[(r, s['step'], s['phase']) for r, s in enumerate(st)]}")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("slots", [1, 3])
def test_dp_reduce_protocol(world, slots):
    for seed in range(8):
        simulate(seed * 17 + world + 100 * slots, world, steps=5, grid=4, max_slots=slots)


def test_model_catches_a_missing_ready_wait(monkeypatch):
    def no_wait(rank, e, world):
        return
        yield

    monkeypatch.setattr(sys.modules[__name__], "wait_ready", no_wait)
    caught = 0
    for seed in range(40):
        try:
            simulate(seed, 3, steps=4, grid=3, max_slots=2)
        except AssertionError:
            caught += 1
    assert caught > 0
