"""Model check of the barrier protocols of the tcgen05 attention backward
(``nano_megatron_b200/csrc/attention_bwd_tc.cu``), on the CPU.

Every role of each kernel (TMA producer, MMA issuer, elementwise warpgroups)
is a coroutine that issues the same waits, arrives, MMAs and commits as the
kernel, in the kernel's order. Three engines stand in for the hardware:

* mbarriers with PTX parity semantics: ``try_wait.parity(P)`` succeeds when the
  barrier's current phase parity differs from ``P``;
* the tensor core executes MMAs in issue order, and a commit arrives on its
  barrier once every MMA issued before it has executed;
* TMA loads land after a random delay.

A random scheduler interleaves them. Each run checks that

* no waiter ever polls a barrier that is more than one phase away from the
  completion it means, so a parity test can neither alias an older completion
  nor miss one (the invariant behind the kernels' "never skips a phase");
* every MMA reads operands (TMEM columns, ring slots) written for its block and
  not yet overwritten, and every overwrite comes after the last reader of the
  previous contents executed;
* every role finishes (no deadlock) for block counts from 1 up, and the dQ and
  dK / dV accumulations run in block order.

Variants with one rule of the protocol removed must be caught, so the checks
are not vacuous.
"""

import random

import pytest

from tests._kernel_constants import constant

Q_STAGES = constant("attention_bwd_tc.cu", "Q_STAGES")
KV_STAGES = constant("attention_bwd_tc.cu", "KV_STAGES")


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.completed = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.completed += 1
            self.pending = self.count

    def poll(self, k):
        """Poll for completion ``k`` (0-based) with the parity the kernel uses."""
        assert self.completed in (k, k + 1), (
            f"{self.name}: waiting for completion {k} while {self.completed} completed: the parity would "
            f"{'alias an older phase' if self.completed < k else 'miss this one'}")
        return (self.completed & 1) != (k & 1)


class Machine:
    """Barriers, an in-order tensor core with commits, and delayed TMA."""

    def __init__(self, rng):
        self.rng = rng
        self.mma_queue = []  # issued, not executed: ("mma", fn) or ("commit", barrier)
        self.tma = []        # in flight: [remaining delay, fn]

    @staticmethod
    def bar(name, count=1):
        return Barrier(name, count)

    def issue(self, fn):
        self.mma_queue.append(("mma", fn))

    def commit(self, barrier):
        self.mma_queue.append(("commit", barrier))

    def load(self, fn):
        self.tma.append([self.rng.randint(1, 12), fn])

    def engines_step(self):
        if self.mma_queue and self.rng.random() < 0.5:
            kind, x = self.mma_queue.pop(0)
            x() if kind == "mma" else x.arrive()
        for t in self.tma:
            t[0] -= 1
        landed = [t for t in self.tma if t[0] <= 0]
        self.tma = [t for t in self.tma if t[0] > 0]
        for t in landed:
            t[1]()


def wait(barrier, k):
    """Yield until completion ``k`` of ``barrier`` has happened."""
    while not barrier.poll(k):
        yield


def run(machine, roles, max_steps=100000):
    live = list(roles)
    for _ in range(max_steps):
        if not live and not machine.mma_queue and not machine.tma:
            return
        machine.engines_step()
        if live:
            r = machine.rng.choice(live)
            try:
                next(r)
            except StopIteration:
                live.remove(r)
    raise AssertionError(f"deadlock: {len(live)} roles still waiting")


# ---------------------------------------------------------------- dQ kernel
def dq_kernel(rng, nblk, stages=Q_STAGES, broken=None):
    """128-key blocks, both groups on every block, separate S and dP hand-offs,
    dS in columns of its own, Q staged in the V slot of stage 2 until copied
    into TMEM. ``broken``: "s_free" issues S(j+1) without waiting for both
    groups to load S(j); "ds_empty" stores dS(j) without waiting for dQ(j-1)."""
    m = Machine(rng)
    qdo_full, q_tmem, acc_done = m.bar("qdo_full"), m.bar("q_tmem"), m.bar("acc_done")
    kv_full = [m.bar(f"kv_full{i}") for i in range(stages)]
    kv_empty = [m.bar(f"kv_empty{i}") for i in range(stages)]
    s_full, dp_full, ds_empty = m.bar("s_full"), m.bar("dp_full"), m.bar("ds_empty")
    s_free, dp_free, ds_full = m.bar("s_free", 2), m.bar("dp_free", 2), m.bar("ds_full", 2)
    slot = {2: "Q"}                  # stage -> block whose K/V it holds
    s_cols = dp_cols = None          # block whose S / dP the columns hold
    ds_half = [None, None]           # block whose dS each group's half of the dS columns holds
    loaded_s, loaded_dp = set(), set()
    dq_done = []

    def producer():
        m.load(qdo_full.arrive)
        for j in range(nblk):
            st = j % stages
            if j >= stages:
                yield from wait(kv_empty[st], j // stages - 1)
            if j == 2:
                yield from wait(q_tmem, 0)
            assert slot.get(st) in (None, "Q", j - stages), "K/V slot refilled before its last reader"

            def land(st=st, j=j):
                slot[st] = j
                kv_full[st].arrive()
            m.load(land)
            yield

    def mma():
        yield from wait(qdo_full, 0)
        yield from wait(q_tmem, 0)
        ns = nd = na = 0
        while na < nblk:
            if na < nd and ds_full.poll(na):
                j, st = na, na % stages

                def dq(j=j, st=st):
                    assert slot[st] == j, "dQ read a K block that was replaced"
                    assert ds_half == [j, j], "dQ read dS that was not (or no longer) block j"
                    dq_done.append(j)
                m.issue(dq)
                m.commit(kv_empty[st])
                m.commit(ds_empty)
                na += 1
            if ns < nblk and ns <= nd and (ns == 0 or broken == "s_free" or s_free.poll(ns - 1)):
                st = ns % stages
                if kv_full[st].poll(ns // stages):
                    def s_mma(j=ns, st=st):
                        nonlocal s_cols
                        assert slot[st] == j
                        assert j == 0 or {(j - 1, 0), (j - 1, 1)} <= loaded_s, "S overwritten before both loads"
                        s_cols = j
                    m.issue(s_mma)
                    m.commit(s_full)
                    ns += 1
            if nd < ns and (nd == 0 or dp_free.poll(nd - 1)):
                def dp_mma(j=nd, st=nd % stages):
                    nonlocal dp_cols
                    assert slot[st] == j
                    assert j == 0 or {(j - 1, 0), (j - 1, 1)} <= loaded_dp, "dP overwritten before both loads"
                    dp_cols = j
                m.issue(dp_mma)
                m.commit(dp_full)
                nd += 1
            yield
        m.commit(acc_done)

    def group(g):
        if g == 0:
            yield from wait(qdo_full, 0)
            q_tmem.arrive()
        for j in range(nblk):
            yield from wait(s_full, j)
            assert s_cols == j, "loaded S of another block"
            loaded_s.add((j, g))
            s_free.arrive()
            yield
            yield from wait(dp_full, j)
            assert dp_cols == j, "loaded dP of another block"
            loaded_dp.add((j, g))
            dp_free.arrive()
            yield
            if j > 0 and broken != "ds_empty":
                yield from wait(ds_empty, j - 1)
            assert j == 0 or (j - 1) in dq_done, "dS stored over a block dQ had not read"
            ds_half[g] = j
            ds_full.arrive()
        yield from wait(acc_done, 0)

    run(m, [producer(), mma(), group(0), group(1)])
    assert dq_done == list(range(nblk))


# ------------------------------------------------------------ dK / dV kernel
def dkdv_kernel(rng, nblk, stages=KV_STAGES, ahead=2):
    """64-query blocks taken alternately by two groups, each with its own
    S^T/dP^T columns (P^T/dS^T written over them); S^T/dP^T of block ns are
    issued while ns < na + ``ahead`` (the kernel uses 2: the same group's
    previous block must have had its dV/dK products issued)."""
    m = Machine(rng)
    kv_full, acc_done = m.bar("kv_full"), m.bar("acc_done")
    qdo_full = [m.bar(f"qdo_full{i}") for i in range(stages)]
    qdo_empty = [m.bar(f"qdo_empty{i}") for i in range(stages)]
    st_full = [m.bar(f"st_full{g}") for g in range(2)]
    pds_full = [m.bar(f"pds_full{g}", 1) for g in range(2)]
    slot = {}
    cols = [None, None]   # group -> block whose S^T/dP^T (then P^T/dS^T) its columns hold
    written = set()       # blocks whose P^T/dS^T are in TMEM
    acc_done_blocks = []

    def producer():
        m.load(kv_full.arrive)
        for i in range(nblk):
            st = i % stages
            if i >= stages:
                yield from wait(qdo_empty[st], i // stages - 1)
            assert slot.get(st) in (None, i - stages), "Q/dO slot refilled before its last reader"

            def land(st=st, i=i):
                slot[st] = i
                qdo_full[st].arrive()
            m.load(land)
            yield

    def mma():
        yield from wait(kv_full, 0)
        ns = na = 0
        while na < nblk:
            if ns < nblk and ns < na + ahead:
                g, st = ns & 1, ns % stages
                if qdo_full[st].poll(ns // stages):
                    def sdp(j=ns, g=g, st=st):
                        assert slot[st] == j
                        prev = cols[g]
                        assert prev is None or prev in acc_done_blocks, \
                            "S^T/dP^T overwrote P^T/dS^T before dV/dK read them"
                        cols[g] = j
                    m.issue(sdp)
                    m.commit(st_full[g])
                    ns += 1
            if na < ns:
                g, st = na & 1, na % stages
                if pds_full[g].poll(na >> 1):
                    def dvdk(j=na, g=g, st=st):
                        assert slot[st] == j and cols[g] == j and j in written
                        acc_done_blocks.append(j)
                    m.issue(dvdk)
                    m.commit(qdo_empty[st])
                    na += 1
            yield
        m.commit(acc_done)

    def group(g):
        for n, i in enumerate(range(g, nblk, 2)):
            yield from wait(st_full[g], n)
            assert cols[g] == i, "loaded S^T/dP^T of another block"
            yield
            written.add(i)
            pds_full[g].arrive()
        yield from wait(acc_done, 0)

    run(m, [producer(), mma(), group(0), group(1)])
    assert acc_done_blocks == list(range(nblk))


@pytest.mark.parametrize("nblk", [1, 2, 3, 4, 5, 7, 12])
def test_dq_kernel_protocol(nblk):
    for seed in range(30):
        dq_kernel(random.Random(1000 * nblk + seed), nblk)


@pytest.mark.parametrize("nblk", [1, 2, 3, 4, 5, 6, 9, 16])
def test_dkdv_kernel_protocol(nblk):
    for seed in range(30):
        dkdv_kernel(random.Random(2000 * nblk + seed), nblk)


@pytest.mark.parametrize("variant", [
    lambda rng: dq_kernel(rng, 8, broken="s_free"),
    lambda rng: dq_kernel(rng, 8, broken="ds_empty"),
    lambda rng: dkdv_kernel(rng, 8, ahead=3),
], ids=["dq-without-s_free", "dq-without-ds_empty", "dkdv-three-ahead"])
def test_checker_catches_a_broken_protocol(variant):
    caught = 0
    for seed in range(60):
        try:
            variant(random.Random(seed))
        except AssertionError:
            caught += 1
    assert caught > 0, "a protocol with a rule removed passed every interleaving"
