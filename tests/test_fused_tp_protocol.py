"""Model check of the cross-rank protocol of the fused tensor-parallel kernels
(``nano_megatron_b200/csrc/fused_tp.cu``), on the CPU, with adversarial
scheduling.

Each rank runs a sequence of fused calls on one stream (all-gather -> GEMM and
GEMM -> reduce-scatter, alternating or back to back, new epoch per call, one
shared workspace).
A call is a grid of CTAs; each CTA runs the kernel's comm role and its
producer / epilogue role as coroutines that issue the kernel's flag writes,
flag waits, peer stores and work claims in the kernel's order:

* every CTA announces ``ready[r] = epoch`` on every peer;
* all-gather: push jobs (slice x destination, destination-major) and tiles
  (own chunk first) are claimed from per-rank counters of the epoch's parity,
  which each CTA zeroes for the other parity; a push into peer p waits for
  p's ready, then sets ``ag_done[r][slice]`` on p; a tile of chunk c waits for
  all of c's ``ag_done`` flags and reads the gathered rows;
* reduce-scatter: foreign chunks first, own chunk last; a foreign tile waits
  for the owner's ready, stores its partial into the owner's slot and sets
  ``rs_done``; an own tile waits for every peer's ``rs_done`` and sums.

Residency is adversarial: other kernels (the NCCL or data-parallel work the
kernels share the GPU with) hold a random, changing number of each rank's SM
slots, down to one, and CTAs are dispatched in block order into free slots.
Ranks run at different speeds and reach their calls at different times.
The checks: every call of every rank finishes (no wait depends on a
particular CTA of a peer being resident), every gathered row and every summed
partial read is the current call's data from the right rank (workspace reuse
across calls never lets a fast rank overwrite what a slow one still reads),
and every tile is computed exactly once per call.

Inside a CTA, the producer hands claimed tiles to the MMA warp and the
epilogue through a small queue (``qfull`` / ``qempty`` with two consumers,
then a double-buffered ``ep_tile`` and a named barrier for the epilogue
warps); ``test_tile_queue`` checks that no queue slot or ``ep_tile`` entry is
overwritten before every reader saw it and that both consumers see the claimed
sequence.
"""

import random
import sys

import pytest

from tests._kernel_constants import constant

K_QUEUE = constant("fused_tp.cu", "kQueue")

AG, RS = "ag", "rs"


class Rank:
    def __init__(self, r, world, slices, tiles_per_chunk):
        self.r = r
        self.ready = [0] * world                            # ready[p]: epoch peer p announced here
        self.ag_done = [[0] * slices for _ in range(world)]  # [chunk][slice]
        self.rs_done = [[0] * world for _ in range(tiles_per_chunk)]  # [local tile][source]
        self.gather = [[None] * slices for _ in range(world)]  # [chunk][slice] -> (epoch, chunk, slice)
        self.recv = [[None] * tiles_per_chunk for _ in range(world)]  # [source][local tile]
        self.ctr = {(k, par): 0 for k in ("tiles", "push") for par in (0, 1)}
        self.done_tiles = {}                                 # epoch -> tiles computed


def wait_until(cond):
    while not cond():
        yield


def cta(rank, ranks, epoch, mode, b, world, slices, tiles_per_chunk, log):
    """One CTA: returns its coroutines (comm, worker)."""
    r = rank.r
    par = epoch & 1
    # prologue: zero the other parity's counters, announce the epoch
    rank.ctr[("tiles", 1 - par)] = 0
    rank.ctr[("push", 1 - par)] = 0
    for p in range(world):
        if p != r:
            ranks[p].ready[r] = max(ranks[p].ready[r], epoch)

    def claim(kind):
        v = rank.ctr[(kind, par)]
        rank.ctr[(kind, par)] = v + 1
        return v

    def comm():
        if mode != AG:
            return
        dests = world - 1
        while True:
            job = claim("push")
            if job >= dests * slices:
                return
            d, s = divmod(job, slices)
            p = (r - 1 - d) % world
            yield from wait_until(lambda p=p: rank.ready[p] >= epoch)
            yield
            ranks[p].gather[r][s] = (epoch, r, s)   # the pushed rows (plain peer stores)
            yield
            ranks[p].ag_done[r][s] = epoch          # release after a system fence

    def worker():
        n_tiles = world * tiles_per_chunk
        ready_seen = set()
        while True:
            t = claim("tiles")
            if t >= n_tiles:
                return
            slot, local = divmod(t, tiles_per_chunk)
            if mode == AG:
                chunk = (r + slot) % world
                if chunk != r:
                    yield from wait_until(lambda c=chunk: all(f >= epoch for f in rank.ag_done[c]))
                    for s in range(slices):
                        assert rank.gather[chunk][s] == (epoch, chunk, s), \
                            f"rank {r} epoch {epoch}: gathered rows of chunk {chunk} are {rank.gather[chunk][s]}"
                yield
            else:
                chunk = (r + 1 + slot) % world
                if chunk != r:
                    if chunk not in ready_seen:
                        yield from wait_until(lambda c=chunk: rank.ready[c] >= epoch)
                        ready_seen.add(chunk)
                    yield
                    ranks[chunk].recv[r][local] = (epoch, r, local)
                    yield
                    ranks[chunk].rs_done[local][r] = epoch
                else:
                    yield from wait_until(lambda: all(rank.rs_done[local][s] >= epoch
                                                      for s in range(world) if s != r))
                    for s in range(world):
                        if s != r:
                            assert rank.recv[s][local] == (epoch, s, local), \
                                f"rank {r} epoch {epoch}: partial from {s} for tile {local} is {rank.recv[s][local]}"
            done = rank.done_tiles.setdefault(epoch, [])
            assert (chunk, local) not in done, "tile computed twice"
            done.append((chunk, local))

    return [comm(), worker()]


def simulate(seed, world, modes, slices, tiles_per_chunk, max_slots):
    rng = random.Random(seed)
    ranks = [Rank(r, world, slices, tiles_per_chunk) for r in range(world)]
    calls = len(modes)
    state = [{"call": 0, "next_block": 0, "resident": [], "held": 0} for _ in range(world)]
    speed = [rng.uniform(0.3, 1.0) for _ in range(world)]
    log = []
    for _ in range(400000):
        if all(st["call"] == calls for st in state):
            break
        r = rng.randrange(world)
        st, rank = state[r], ranks[r]
        if st["call"] == calls or rng.random() > speed[r]:
            continue
        # other kernels take or give back SM slots (never all of them)
        if rng.random() < 0.05:
            st["held"] = rng.randint(0, max_slots - 1)
        epoch = st["call"] + 1
        mode = modes[st["call"]]
        # dispatch CTAs in block order into free slots
        while st["next_block"] < slices and len(st["resident"]) < max_slots - st["held"]:
            st["resident"].append(cta(rank, ranks, epoch, mode, st["next_block"], world, slices,
                                      tiles_per_chunk, log))
            st["next_block"] += 1
        if st["resident"]:
            c = rng.choice(st["resident"])
            coro = rng.choice(c)
            try:
                next(coro)
            except StopIteration:
                c.remove(coro)
            if not c:
                st["resident"].remove(c)
        if not st["resident"] and st["next_block"] == slices:
            tiles = rank.done_tiles.get(epoch, [])
            assert sorted(tiles) == sorted((ch, lo) for ch in range(world) for lo in range(tiles_per_chunk)), \
                f"rank {r} epoch {epoch}: tiles {sorted(tiles)}"
            st["call"] += 1
            st["next_block"] = 0
    stuck = [(r, st["call"]) for r, st in enumerate(state) if st["call"] < calls]
    assert not stuck, f"ranks stuck at calls {stuck}"


SEQUENCES = {
    "alternating": [AG, RS, AG, RS, AG, RS],      # a layer's forward: QKV, out proj, gate|up, down
    "back-to-back": [AG, AG, AG, RS, RS, RS, AG, RS],
}


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("slots", [1, 2, 5])
@pytest.mark.parametrize("seq", sorted(SEQUENCES))
def test_fused_tp_protocol_completes_under_partial_residency(world, slots, seq):
    for seed in range(6):
        simulate(seed * 131 + world * 7 + slots, world, SEQUENCES[seq], slices=5, tiles_per_chunk=3,
                 max_slots=slots)


def test_model_catches_a_missing_ready_wait(monkeypatch):
    """Without the wait for the peer's ready flag, a fast rank overwrites the
    gather rows a slow rank is still reading: the check must see it."""
    orig = wait_until

    def skip_ready(cond):
        # drop the ready waits (they are the only waits on `ready`), keep the others
        if "ready" in cond.__code__.co_names:
            return
        yield from orig(cond)

    monkeypatch.setattr(sys.modules[__name__], "wait_until", skip_ready)
    caught = 0
    for seed in range(40):
        try:
            simulate(seed, 3, SEQUENCES["back-to-back"], slices=4, tiles_per_chunk=2, max_slots=2)
        except AssertionError:
            caught += 1
    assert caught > 0


# ------------------------------------------------- intra-CTA tile queue
class QBarrier:
    def __init__(self, name, count=1):
        self.name, self.count, self.pending, self.completed = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.completed += 1
            self.pending = self.count

    def poll(self, k):
        assert self.completed in (k, k + 1), f"{self.name}: waiting for completion {k}, {self.completed} completed"
        return (self.completed & 1) != (k & 1)


def queue_cta(seed, claims, queue=K_QUEUE, warps=4, broken=None):
    """The producer hands claimed tiles (then -1) through a ``queue``-slot ring
    to the MMA warp and the epilogue leader (``qempty`` expects both); the
    leader passes each to the epilogue warps through ``ep_tile[it & 1]`` and a
    named barrier per iteration. ``broken``: "one_consumer" arms qempty for one
    arrival; "single_ep_tile" uses one ep_tile entry."""
    rng = random.Random(seed)
    qfull = [QBarrier(f"qfull{s}") for s in range(queue)]
    qempty = [QBarrier(f"qempty{s}", 1 if broken == "one_consumer" else 2) for s in range(queue)]
    tq = [None] * queue
    readers = [set() for _ in range(queue)]   # who read the current content of a slot
    ep_tile, ep_seen = [None, None], [set(), set()]
    got = {"mma": [], "ep": [[] for _ in range(warps)]}
    arrived = [0]                              # named barrier: arrivals of the current generation
    generation = [0]

    def wait(bar, k):
        while not bar.poll(k):
            yield

    def producer():
        for it, t in enumerate(claims + [-1]):
            s = it % queue
            if it >= queue:
                yield from wait(qempty[s], it // queue - 1)
            assert tq[s] is None or readers[s] >= {"mma", "ep"}, f"queue slot {s} overwritten before both read it"
            tq[s], readers[s] = t, set()
            qfull[s].arrive()
            yield

    def mma():
        for it in range(len(claims) + 1):
            s = it % queue
            yield from wait(qfull[s], it // queue)
            t = tq[s]
            readers[s].add("mma")
            qempty[s].arrive()
            if t < 0:
                return
            got["mma"].append(t)
            yield

    def bar_sync():
        gen = generation[0]
        arrived[0] += 1
        if arrived[0] == warps:
            arrived[0] = 0
            generation[0] += 1
        while generation[0] == gen:
            yield

    def epilogue(w):
        for it in range(len(claims) + 1):
            b = 0 if broken == "single_ep_tile" else it & 1
            if w == 0:
                s = it % queue
                yield from wait(qfull[s], it // queue)
                nxt = tq[s]
                readers[s].add("ep")
                qempty[s].arrive()
                assert ep_tile[b] is None or ep_seen[b] == set(range(warps)), "ep_tile overwritten before every warp read it"
                ep_tile[b], ep_seen[b] = nxt, set()
            yield from bar_sync()
            t = ep_tile[b]
            ep_seen[b].add(w)
            if t < 0:
                return
            got["ep"][w].append(t)
            yield

    roles = [producer(), mma()] + [epilogue(w) for w in range(warps)]
    for _ in range(100000):
        if not roles:
            break
        r = rng.choice(roles)
        try:
            next(r)
        except StopIteration:
            roles.remove(r)
    assert not roles, "the queue deadlocked"
    assert got["mma"] == claims and all(g == claims for g in got["ep"])


@pytest.mark.parametrize("n", [0, 1, 3, 4, 9, 17])
def test_tile_queue(n):
    for seed in range(30):
        queue_cta(seed, list(range(10, 10 + n)))


@pytest.mark.parametrize("broken", ["one_consumer", "single_ep_tile"])
def test_tile_queue_checker_catches_a_broken_protocol(broken):
    caught = 0
    for seed in range(40):
        try:
            queue_cta(seed, list(range(12)), broken=broken)
        except AssertionError:
            caught += 1
    assert caught > 0
