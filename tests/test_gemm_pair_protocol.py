"""Model check of the CTA-pair handshake of the tcgen05 GEMM
(``nano_megatron_b200/csrc/gemm.cu``, ``PAIR``), on the CPU.

A pair is two CTAs of a cluster; CTA 0 (the leader) issues every MMA, which
reads a stage of both CTAs' shared memory and writes both CTAs' TMEM:

* each CTA's producer waits for its own ``empty[stage]``; the leader arms its
  ``full[stage]`` with the byte count of both CTAs' loads, and the loads of
  both CTAs complete their bytes on the leader's ``full[stage]`` (a load of
  CTA 1 may land before the leader armed the phase: the transaction count
  goes negative for a while, as the hardware allows);
* the leader waits for ``full[stage]``, issues the stage's MMAs and a commit
  multicast to ``empty[stage]`` of both CTAs; after a tile's k-blocks a commit
  multicast to ``tfull[acc]`` of both CTAs (two accumulators);
* each CTA's four epilogue warps wait for their own ``tfull[acc]``, read their
  TMEM rows and arrive on the leader's ``tempty[acc]`` (8 arrivals), which the
  leader waits for before reusing the accumulator.

Random interleavings check: the parity of every wait stays within one phase of
the completion it means, no stage or accumulator is overwritten before its
reader ran, every (tile, k-block) is multiplied once and in order, and the pair
finishes. Variants with one rule broken are caught.
"""

import random

import pytest

from tests._kernel_constants import constant

PAIR_STAGES = constant("gemm.cu", "PAIR_STAGES")


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.tx, self.completed = name, count, count, 0, 0

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.completed += 1
            self.pending = self.count

    def arrive(self, expect_tx=0):
        self.tx += expect_tx
        self.pending -= 1
        assert self.pending >= 0
        self._check()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._check()

    def poll(self, k):
        assert self.completed in (k, k + 1), f"{self.name}: waiting for completion {k}, {self.completed} completed"
        return (self.completed & 1) != (k & 1)


def wait(bar, k):
    while not bar.poll(k):
        yield


def simulate(seed, units, kblocks, stages, broken=None):
    """``broken``: "early_release" (epilogue warps arrive on tempty before
    reading TMEM), "no_empty_wait" (CTA 1's producer refills a stage without
    waiting for its empty barrier), "half_tx" (the leader arms full[stage]
    with its own half's bytes only)."""
    rng = random.Random(seed)
    SB = 2  # bytes of one CTA's half of a stage (two loads of 1)
    full = [[Barrier(f"full{c}.{s}", 1) for s in range(stages)] for c in range(2)]
    empty = [[Barrier(f"empty{c}.{s}", 1) for s in range(stages)] for c in range(2)]
    tfull = [[Barrier(f"tfull{c}.{a}", 1) for a in range(2)] for c in range(2)]
    tempty = [Barrier(f"tempty{a}", 8) for a in range(2)]  # on the leader
    smem = [[None] * stages for _ in range(2)]   # CTA -> stage -> (unit, kb) it holds
    acc = [[None] * 2 for _ in range(2)]         # CTA -> accumulator -> (unit, k-blocks done)
    read_back = [[None] * 2 for _ in range(2)]   # CTA -> accumulator -> unit whose result was read
    mma_queue, tma = [], []
    multiplied = []

    def commit_multicast(bars):
        mma_queue.append(("commit", bars))

    def producer(c):
        stage_uses = [0] * stages
        i = 0
        for u in range(units):
            for kb in range(kblocks):
                s = i % stages
                if stage_uses[s] > 0 and not (broken == "no_empty_wait" and c == 1):
                    yield from wait(empty[c][s], stage_uses[s] - 1)
                assert smem[c][s] is None or smem[c][s][2], f"CTA {c} stage {s} refilled before the MMA read it"
                stage_uses[s] += 1
                if c == 0:
                    full[0][s].arrive(expect_tx=SB if broken == "half_tx" else 2 * SB)
                yield
                for _ in range(2):  # two boxes per CTA half
                    def land(c=c, s=s, u=u, kb=kb):
                        if smem[c][s] is None or smem[c][s][:2] != (u, kb):
                            smem[c][s] = (u, kb, False)
                        full[0][s].complete_tx(1)
                    tma.append([rng.randint(1, 10), land])
                i += 1

    def mma():
        stage_uses = [0] * stages
        acc_uses = [0, 0]
        i = 0
        for u in range(units):
            a = u & 1
            if acc_uses[a] > 0:
                yield from wait(tempty[a], acc_uses[a] - 1)
            acc_uses[a] += 1
            for kb in range(kblocks):
                s = i % stages
                yield from wait(full[0][s], stage_uses[s])
                stage_uses[s] += 1

                def exe(s=s, u=u, kb=kb, a=a):
                    for c in range(2):
                        assert smem[c][s] is not None and smem[c][s][:2] == (u, kb), \
                            f"MMA of ({u}, {kb}) read CTA {c} stage {s} holding {smem[c][s]}"
                        if kb == 0:
                            assert acc[c][a] is None or read_back[c][a] == acc[c][a][0], \
                                f"accumulator {a} of CTA {c} overwritten before its epilogue read it"
                            acc[c][a] = (u, 0)
                        assert acc[c][a] == (u, kb)
                        acc[c][a] = (u, kb + 1)
                    multiplied.append((u, kb))
                mma_queue.append(("mma", exe))

                def consumed(s=s):
                    for c in range(2):
                        smem[c][s] = smem[c][s][:2] + (True,)
                mma_queue.append(("mma", consumed))
                commit_multicast([empty[0][s], empty[1][s]])
                i += 1
                yield
            commit_multicast([tfull[0][a], tfull[1][a]])

    def epilogue(c, w):
        uses = [0, 0]
        for u in range(units):
            a = u & 1
            yield from wait(tfull[c][a], uses[a])
            uses[a] += 1
            if broken == "early_release":
                tempty[a].arrive()
                yield
            assert acc[c][a] == (u, kblocks), f"CTA {c} read accumulator {a} holding {acc[c][a]}"
            yield
            if w == 0:
                read_back[c][a] = u
            if broken != "early_release":
                tempty[a].arrive()  # remote arrive on the leader's barrier for CTA 1

    roles = [producer(0), producer(1), mma()] + [epilogue(c, w) for c in range(2) for w in range(4)]
    for _ in range(200000):
        if not roles and not mma_queue and not tma:
            break
        if mma_queue and rng.random() < 0.5:
            kind, x = mma_queue.pop(0)
            if kind == "mma":
                x()
            else:
                for b in x:
                    b.arrive()
        for t in tma:
            t[0] -= 1
        for t in [t for t in tma if t[0] <= 0]:
            tma.remove(t)
            t[1]()
        if roles:
            r = rng.choice(roles)
            try:
                next(r)
            except StopIteration:
                roles.remove(r)
    assert not roles and not mma_queue and not tma, "the pair did not finish"
    assert multiplied == [(u, kb) for u in range(units) for kb in range(kblocks)]


@pytest.mark.parametrize("units,kblocks,stages", [(1, 1, PAIR_STAGES), (3, 2, PAIR_STAGES), (5, 7, PAIR_STAGES),
                                                  (4, 13, PAIR_STAGES), (6, 3, 2)])
def test_gemm_pair_handshake(units, kblocks, stages):
    for seed in range(25):
        simulate(seed + 31 * units + kblocks, units, kblocks, stages)


@pytest.mark.parametrize("broken", ["early_release", "no_empty_wait", "half_tx"])
def test_checker_catches_a_broken_handshake(broken):
    caught = 0
    for seed in range(40):
        try:
            simulate(seed, 6, 4, 3, broken=broken)
        except AssertionError:
            caught += 1
    assert caught > 0, f"{broken} passed every interleaving"
