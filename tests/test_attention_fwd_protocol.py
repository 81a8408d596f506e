"""Model check of the barrier protocol of the tcgen05 attention forward
(``nano_megatron_b200/csrc/attention_tc.cu``), on the CPU.

One CTA holds two 128-row query tiles. Roles, in the kernel's order:

* loads: Q once; K_j and V_j through two-slot rings, each slot refilled after
  its ``k_empty`` / ``v_empty`` commit;
* MMA: QK_0(0), QK_1(0); then for j = 1..: for each tile t, PV_t(j-1) once the
  softmax published P_t(j-1) (``p_full``), then QK_t(j) over the same TMEM
  columns; commits release K slot j after the QKs of block j and V slot j-1
  after the PVs of block j-1;
* softmax of tile t: per block, wait ``s_full[t]``, (maybe rescale O_t, which
  needs PV_t(j-1) complete), write P_t(j) over S_t, arrive ``p_full[t]``; at
  the end arrive ``fin[t]``;
* epilogue: per tile, ``fin[t]`` first, then the last ``pv_done[t]``.

The tensor core runs MMAs in issue order; a commit arrives once every MMA
issued before it ran; TMA lands after a random delay. Random interleavings
check the parity window of every wait, that no S/P columns, O rows, K or V
slot is overwritten before its reader ran, that O_t sums every block once and
in order before the epilogue reads it, and that nothing deadlocks. Variants
with one rule broken are caught.
"""

import random

import pytest


class Barrier:
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


def wait(bar, k):
    while not bar.poll(k):
        yield


def simulate(seed, nkb0, nkb1, broken=None):
    """``broken``: "qk_before_pv" (QK_t(j) issued before PV_t(j-1)),
    "no_k_empty" (K slots refilled without waiting), "pv_only" (the epilogue
    waits for the last pv_done without fin first)."""
    rng = random.Random(seed)
    nkb = [nkb0, nkb1]
    nkb_max = max(nkb)
    q_full, mma_done = Barrier("q_full"), Barrier("mma_done")
    k_full = [Barrier(f"k_full{s}") for s in range(2)]
    v_full = [Barrier(f"v_full{s}") for s in range(2)]
    k_empty = [Barrier(f"k_empty{s}") for s in range(2)]
    v_empty = [Barrier(f"v_empty{s}") for s in range(2)]
    s_full = [Barrier(f"s_full{t}") for t in range(2)]
    pv_done = [Barrier(f"pv_done{t}") for t in range(2)]
    p_full = [Barrier(f"p_full{t}", 4) for t in range(2)]  # one arrival per softmax warp
    fin = [Barrier(f"fin{t}", 4) for t in range(2)]
    k_slot, v_slot = [None, None], [None, None]            # block each slot holds (+ read marks)
    k_read, v_read = set(), set()
    sp = [None, None]      # tile -> ("S", j) or ("P", j) in its TMEM columns
    o = [[], []]           # tile -> blocks accumulated into O_t
    o_read = [False, False]
    mma_q, tma = [], []

    def issue(fn):
        mma_q.append(("mma", fn))

    def commit(bar):
        mma_q.append(("commit", bar))

    def loader():
        tma.append([rng.randint(1, 8), q_full.arrive])
        for j in range(nkb_max):
            st = j & 1
            if j >= 2 and broken != "no_k_empty":
                yield from wait(k_empty[st], (j >> 1) - 1)
            assert j < 2 or (j - 2) in k_read, "K slot refilled before its QK products read it"

            def land_k(st=st, j=j):
                k_slot[st] = j
                k_full[st].arrive()
            tma.append([rng.randint(1, 8), land_k])
            yield
            if j >= 2:
                yield from wait(v_empty[st], (j >> 1) - 1)
            assert j < 2 or (j - 2) in v_read, "V slot refilled before its PV products read it"

            def land_v(st=st, j=j):
                v_slot[st] = j
                v_full[st].arrive()
            tma.append([rng.randint(1, 8), land_v])
            yield

    def qk(t, j):
        def run():
            assert k_slot[j & 1] == j, "QK read the wrong K block"
            assert sp[t] is None or sp[t] == ("P", j - 1) and (j - 1) in o[t], \
                f"QK_{t}({j}) overwrote {sp[t]} before PV read it"
            sp[t] = ("S", j)
            if t == 1 or nkb[1] <= j:
                k_read.add(j)
        issue(run)
        commit(s_full[t])

    def pv(t, i):
        def run():
            assert sp[t] == ("P", i), f"PV_{t}({i}) read {sp[t]}"
            assert v_slot[i & 1] == i
            assert o[t] == list(range(i)) and not o_read[t]
            o[t].append(i)
        issue(run)
        commit(pv_done[t])

    def mma():
        yield from wait(q_full, 0)
        yield from wait(k_full[0], 0)
        qk(0, 0)
        if nkb[1] > 0:
            qk(1, 0)
        commit(k_empty[0])
        for j in range(1, nkb_max + 1):
            i = j - 1
            if j < nkb_max:
                yield from wait(k_full[j & 1], j >> 1)  # the kernel polls this completion's parity
            yield from wait(v_full[i & 1], i >> 1)
            for t in range(2):
                order = ["qk", "pv"] if broken == "qk_before_pv" else ["pv", "qk"]
                for step in order:
                    if step == "pv" and i < nkb[t]:
                        yield from wait(p_full[t], i)
                        pv(t, i)
                    if step == "qk" and j < nkb[t]:
                        qk(t, j)
                if t == 1:
                    mma_q.append(("mma", lambda i=i: v_read.add(i)))
                    commit(v_empty[i & 1])
            if j < nkb_max:
                commit(k_empty[j & 1])
            yield
        commit(mma_done)

    def softmax(t, w):
        for j in range(nkb[t]):
            yield from wait(s_full[t], j)
            assert sp[t] in (("S", j), ("P", j)), f"softmax {t} block {j} sees {sp[t]}"
            if j > 0:
                assert o[t] == list(range(j)), "O rescaled before PV of the previous block completed"
            yield
            if w == 0:
                sp[t] = ("P", j)
            p_full[t].arrive()
        if nkb[t] > 0:
            fin[t].arrive()

    def epilogue():
        for t in range(2):
            if nkb[t] == 0:
                continue
            if broken != "pv_only":
                yield from wait(fin[t], 0)
            yield from wait(pv_done[t], nkb[t] - 1)
            assert o[t] == list(range(nkb[t])), f"epilogue of tile {t} read O after blocks {o[t]}"
            o_read[t] = True
            yield

    roles = [loader(), mma(), epilogue()] + [softmax(t, w) for t in range(2) for w in range(4)]
    for _ in range(200000):
        if not roles and not mma_q and not tma:
            break
        if mma_q and rng.random() < 0.5:
            kind, x = mma_q.pop(0)
            x() if kind == "mma" else x.arrive()
        for item in tma:
            item[0] -= 1
        for item in [x for x in tma if x[0] <= 0]:
            tma.remove(item)
            item[1]()
        if roles:
            r = rng.choice(roles)
            try:
                next(r)
            except StopIteration:
                roles.remove(r)
    assert not roles and not mma_q and not tma, "the CTA did not finish"


@pytest.mark.parametrize("blk", [0, 1, 2, 5])
@pytest.mark.parametrize("second_tile", [True, False])
def test_attention_fwd_protocol(blk, second_tile):
    nkb0 = 2 * blk + 1
    nkb1 = nkb0 + 1 if second_tile else 0
    for seed in range(25):
        simulate(seed + 97 * blk, nkb0, nkb1)


@pytest.mark.parametrize("broken", ["qk_before_pv", "no_k_empty", "pv_only"])
def test_checker_catches_a_broken_protocol(broken):
    caught = 0
    for seed in range(40):
        try:
            simulate(seed, 5, 6, broken=broken)
        except AssertionError:
            caught += 1
    assert caught > 0, f"{broken} passed every interleaving"
