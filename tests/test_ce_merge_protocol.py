"""Model check of the cross-rank protocol of the vocab-parallel cross-entropy
merge (``ce_merge_kernel`` in ``nano_megatron_b200/csrc/fused_tp.cu``), on the
CPU, with adversarial scheduling.

Each rank runs a sequence of merge calls on one stream (one per microbatch of
the last pipeline stage), epoch ``e = 1, 2, ...``. Block ``b`` of rank ``r``:

* writes its rows' (max, sum-exp, target) triples into every rank's data area
  (its own included), slot ``e & 1``, section ``r``;
* after a system fence, sets ``flag[r][b] = e`` on every peer (release);
* waits until ``flag[p][b] >= e`` for every peer ``p`` (acquire, bounded);
* reads every section of its own slot ``e & 1`` and merges.

Ranks run at different speeds; each GPU has a random number of block slots
free (other kernels hold the rest) and dispatches blocks in block order. The
checks: every call of every rank finishes, and every triple a block merges is
the current call's triple from the right rank (the two slots keep a fast rank
from overwriting what a slow rank still reads: a rank that started call
``e + 1`` has seen every peer's flags of call ``e``, so every peer has
finished call ``e - 1``, the previous user of that slot).

Block ``b`` waits only for block ``b`` of each peer, so under partial
residency the protocol relies on blocks being dispatched in index order (the
lowest unfinished index is then resident on every rank); the grid is at most
1024 blocks of 256 threads, which fits on the GPU at once.
``test_dispatch_order_assumption`` shows both halves of that statement.
"""

import random

import pytest


class Rank:
    def __init__(self, r, world, blocks, slots):
        self.r = r
        self.data = [[[None] * blocks for _ in range(world)] for _ in range(slots)]  # [slot][source][block]
        self.flags = [[0] * blocks for _ in range(world)]                             # [source][block]
        self.merged = {}                                                              # epoch -> blocks


def wait_until(cond):
    while not cond():
        yield


def block(rank, ranks, epoch, b, world, slots, broken):
    r = rank.r
    slot = epoch % slots

    def write_data():
        for p in range(world):
            yield
            ranks[p].data[slot][r][b] = (epoch, r, b)

    def write_flags():
        for p in range(world):
            if p != r:
                yield
                ranks[p].flags[r][b] = epoch

    if broken == "flag_before_data":
        yield from write_flags()
        yield from write_data()
    else:
        yield from write_data()
        yield from write_flags()
    for p in range(world):
        if p != r:
            if broken == "equal_wait":
                yield from wait_until(lambda p=p: rank.flags[p][b] == epoch)
            else:
                yield from wait_until(lambda p=p: rank.flags[p][b] >= epoch)
    for p in range(world):
        yield
        got = rank.data[slot][p][b]
        assert got == (epoch, p, b), f"rank {r} call {epoch} block {b}: section {p} holds {got}"
    rank.merged.setdefault(epoch, set()).add(b)


def simulate(seed, world, calls, blocks, max_slots, *, broken=None, in_order=True, steps=300000):
    rng = random.Random(seed)
    slots = 1 if broken == "one_slot" else 2
    ranks = [Rank(r, world, blocks, slots) for r in range(world)]
    state = [{"call": 0, "pending": list(range(blocks)), "resident": [], "held": 0} for _ in range(world)]
    speed = [rng.uniform(0.2, 1.0) for _ in range(world)]
    for _ in range(steps):
        if all(st["call"] == calls for st in state):
            return True
        r = rng.randrange(world)
        st, rank = state[r], ranks[r]
        if st["call"] == calls or rng.random() > speed[r]:
            continue
        if rng.random() < 0.05:  # other kernels take or give back block slots (never all)
            st["held"] = rng.randint(0, max_slots - 1)
        epoch = st["call"] + 1
        while st["pending"] and len(st["resident"]) < max_slots - st["held"]:
            nxt = st["pending"].pop(0 if in_order else rng.randrange(len(st["pending"])))
            st["resident"].append(block(rank, ranks, epoch, nxt, world, slots, broken))
        if st["resident"]:
            coro = rng.choice(st["resident"])
            try:
                next(coro)
            except StopIteration:
                st["resident"].remove(coro)
        if not st["resident"] and not st["pending"]:
            assert rank.merged.get(epoch) == set(range(blocks)), f"rank {r} call {epoch}"
            st["call"] += 1  # stream order: the next call starts after every block of this one
            st["pending"] = list(range(blocks))
    return False


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("max_slots", [1, 2, 6])
def test_ce_merge_completes_with_current_data(world, max_slots):
    for seed in range(8):
        assert simulate(seed * 97 + world * 5 + max_slots, world, calls=6, blocks=4, max_slots=max_slots), \
            f"seed {seed}: ranks did not finish"


@pytest.mark.parametrize("broken", ["one_slot", "flag_before_data", "equal_wait"])
def test_model_catches_a_broken_protocol(broken):
    """One data slot lets a fast rank overwrite a section a slow rank still
    reads; flags before data let a peer read a stale section; an exact-epoch
    wait misses a flag that a peer already moved on to the next call."""
    caught = 0
    for seed in range(60):
        try:
            if not simulate(seed, 3, calls=6, blocks=3, max_slots=3, broken=broken, steps=60000):
                caught += 1
        except AssertionError:
            caught += 1
    assert caught > 0


def test_dispatch_order_assumption():
    """With every block resident, any dispatch order completes; with fewer slots
    than blocks, out-of-order dispatch can leave each rank's resident blocks
    waiting for blocks its peer has not dispatched."""
    for seed in range(10):
        assert simulate(seed, 2, calls=3, blocks=4, max_slots=4, in_order=False)
    stuck = sum(not simulate(seed, 2, calls=3, blocks=4, max_slots=1, in_order=False, steps=40000)
                for seed in range(20))
    assert stuck > 0
