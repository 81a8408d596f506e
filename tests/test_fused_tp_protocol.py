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
"""

import random
import sys

import pytest

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
