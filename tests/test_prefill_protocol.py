"""The one-head tcgen05 prefill kernel's synchronisation protocol
(csrc/prefill_tc.cu, prefill_tc_kernel), modelled on the CPU and run under
randomised adversarial timing.

Actors, as in the kernel: the K producer (warp 0; it issues Q and K(0)
before the CTA barrier), the V producer (warp 6), the MMA issuer (warp 1)
and four softmax warps (warps 2-5, one TMEM lane quarter each); the TMA
engine completes loads in any order after any delay; the tensor pipe runs
the issued MMAs and commits strictly in issue order, a commit arriving on
its mbarrier once everything issued before it has run.  mbarriers keep the
hardware's phase parity: try_wait.parity(P) passes while the current
phase's parity differs from P, so a waiter that fell two phases behind
would be fooled -- the model would then read the wrong tile and fail.

Checked on every run: each Q.K^T reads Q and the K tile it was issued for;
each softmax warp reads S(j) of its own tile and, when it rescales O,
finds every P.V up to j-1 in it; each P.V reads P(i) written by all four
warps and the V tile i; the epilogue finds all P.V products in O; no actor
waits forever.  The softmax warps' lazy-rescale choice (wait for the last
P.V only when some row's maximum moved) is random per warp and tile.

The P-ready barrier is one per parity of the tile, as in the kernel
(p_full[j & 1]); a test shows why ONE barrier is not enough.  The
head-pair kernel (prefill_tc_pair_kernel) is modelled the same way."""
import random

import pytest

STAGES = 2  # kStages of the one-head kernel


class Barrier:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.phase = 0  # completed phases
        self.tx = 0

    def arrive(self):
        self.pending -= 1
        self._maybe_complete()

    def expect_tx(self, n):
        self.tx += n
        self.arrive()

    def complete_tx(self, n):
        self.tx -= n
        self._maybe_complete()

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def test(self, parity):
        return (self.phase & 1) != parity


class Race(AssertionError):
    pass


def run(ntiles, seed, paired_p_full=True):
    """paired_p_full: P(j) arrivals go to p_full[j & 1] (the kernel's
    layout); False models one p_full barrier for every tile."""
    rng = random.Random(seed)
    B = {"q_full": Barrier(1), "pv_done": Barrier(1), "mma_done": Barrier(1)}
    for s in range(2):
        B[f"p_full{s}"] = Barrier(4)

    def pf(j):  # (barrier, parity) that tile j's P arrivals complete
        return (f"p_full{j & 1}", (j >> 1) & 1) if paired_p_full else ("p_full0", j & 1)

    for s in range(STAGES):
        for n in ("k_full", "k_empty", "v_full", "v_empty"):
            B[f"{n}{s}"] = Barrier(1)
    for s in range(2):
        B[f"s_full{s}"] = Barrier(1)
    smem = {"Q": None}
    for s in range(STAGES):
        smem[f"K{s}"] = smem[f"V{s}"] = None
    # S buffers per TMEM lane quarter (softmax warp w owns quarter w):
    # ("S", j) after Q.K^T(j), ("P", j) once warp w wrote its P(j); O: the
    # P.V tiles accumulated in it
    tmem = {"S0": [None] * 4, "S1": [None] * 4, "O": set()}
    tma = []    # pending loads: (region, tile, barrier)
    pipe = []   # issued tensor ops in order

    def load(region, tile, bar):
        B[bar].expect_tx(1)
        tma.append((region, tile, bar))

    # ---------------------------------------------------------------- actors
    # Each actor is a generator that yields a predicate to wait on (or None
    # to just yield the scheduler) and performs its next action once resumed.
    def producer_k():
        load("Q", 0, "q_full")
        load("K0", 0, "k_full0")
        yield None  # the CTA barrier
        for j in range(ntiles):
            if j + 1 < ntiles:
                t = j + 1
                st = t % STAGES
                if t >= STAGES:
                    yield lambda st=st, t=t: B[f"k_empty{st}"].test(((t // STAGES) - 1) & 1)
                load(f"K{st}", t, f"k_full{st}")
            yield None

    def producer_v():
        yield None
        for j in range(ntiles):
            st = j % STAGES
            if j >= STAGES:
                yield lambda st=st, j=j: B[f"v_empty{st}"].test(((j // STAGES) - 1) & 1)
            load(f"V{st}", j, f"v_full{st}")
            yield None

    def issue_pv(i):
        bar, par = pf(i)
        yield lambda: B[bar].test(par)
        st = i % STAGES
        yield lambda: B[f"v_full{st}"].test((i // STAGES) & 1)
        pipe.append(("PV", i, st))
        pipe.append(("commit", "pv_done"))
        pipe.append(("commit", f"v_empty{st}"))

    def mma():
        yield None
        yield lambda: B["q_full"].test(0)
        for j in range(ntiles):
            st = j % STAGES
            yield lambda st=st, j=j: B[f"k_full{st}"].test((j // STAGES) & 1)
            pipe.append(("QK", j, st))
            pipe.append(("commit", f"s_full{j & 1}"))
            pipe.append(("commit", f"k_empty{st}"))
            if j >= 1:
                yield from issue_pv(j - 1)
        yield from issue_pv(ntiles - 1)
        pipe.append(("commit", "mma_done"))
        yield lambda: B["mma_done"].test(0)

    def softmax(w):
        yield None
        for j in range(ntiles):
            sb = j & 1
            yield lambda sb=sb, j=j: B[f"s_full{sb}"].test((j >> 1) & 1)
            got = tmem[f"S{sb}"][w]
            if got != ("S", j):
                raise Race(f"softmax {w} tile {j} read S lanes holding {got}")
            if j >= 1 and rng.random() < 0.3:  # this warp's rows moved their max
                yield lambda j=j: B["pv_done"].test((j - 1) & 1)
                if set(range(j)) - tmem["O"]:
                    raise Race(f"softmax {w} rescaled O before P.V {sorted(set(range(j)) - tmem['O'])}")
            # P(j) over the first columns of S[sb], this warp's lanes
            tmem[f"S{sb}"][w] = ("P", j)
            B[pf(j)[0]].arrive()
            yield None
        yield lambda: B["mma_done"].test(0)
        if tmem["O"] != set(range(ntiles)):
            raise Race(f"epilogue of warp {w} read O with {sorted(tmem['O'])}")

    actors = [producer_k(), producer_v(), mma()] + [softmax(w) for w in range(4)]
    waiting = [None] * len(actors)
    done = [False] * len(actors)

    def step_pipe():
        op = pipe.pop(0)
        if op[0] == "QK":
            _, j, st = op
            if smem["Q"] != 0 or smem[f"K{st}"] != j:
                raise Race(f"Q.K^T({j}) read Q={smem['Q']} K{st}={smem[f'K{st}']}")
            tmem[f"S{j & 1}"] = [("S", j)] * 4
        elif op[0] == "PV":
            _, i, st = op
            p = tmem[f"S{i & 1}"]
            if p != [("P", i)] * 4:
                raise Race(f"P.V({i}) read P lanes holding {p}")
            if smem[f"V{st}"] != i:
                raise Race(f"P.V({i}) read V{st}={smem[f'V{st}']}")
            tmem["O"].add(i)
        else:
            B[op[1]].arrive()

    def step_tma():
        region, tile, bar = tma.pop(rng.randrange(len(tma)))
        smem[region] = tile
        B[bar].complete_tx(1)

    for _ in range(200000):
        choices = []
        for a, gen in enumerate(actors):
            if done[a]:
                continue
            if waiting[a] is None or waiting[a]():
                choices.append(("actor", a))
        if pipe:
            choices.append(("pipe", None))
        if tma:
            choices.append(("tma", None))
        if not choices:
            if all(done):
                return
            raise Race(f"deadlock: waiting actors {[a for a in range(len(actors)) if not done[a]]}")
        kind, a = rng.choice(choices)
        if kind == "pipe":
            step_pipe()
        elif kind == "tma":
            step_tma()
        else:
            try:
                waiting[a] = next(actors[a])
            except StopIteration:
                done[a] = True
    raise Race("no termination")


@pytest.mark.parametrize("ntiles", [1, 2, 3, 4, 5, 8, 13])
def test_prefill_protocol_under_random_timing(ntiles):
    for seed in range(300):
        run(ntiles, seed * 1000 + ntiles)


def test_one_p_full_barrier_lets_a_fast_warp_complete_the_phase_early():
    """With ONE p_full barrier for every tile, a softmax warp that skipped
    its P.V wait (no row of it moved its maximum) runs a whole tile ahead --
    S(j+1) is already there, Q.K^T(j+1) being issued before the MMA warp
    waits for P(j) -- and its arrival for tile j+1 completes tile j's
    four-arrival phase while a slow warp's P(j) lanes still hold scores:
    P.V(j) reads them.  (Holding each arrival until the previous phase
    completed instead still lets the MMA warp miss a phase: two phases can
    complete before it polls, and the parity cannot tell them apart.)"""
    caught = []
    for seed in range(300):
        try:
            run(5, seed, paired_p_full=False)
        except Race as e:
            caught.append(str(e))
    assert any("P.V(" in c and "read P lanes" in c for c in caught), caught[:3]


def run_pair(ntiles, seed, cross_wait=True):
    """The head-pair kernel (prefill_tc_pair_kernel): two heads over shared
    K/V tiles, one S buffer per head (s_full / s_free), ONE shared-memory P
    buffer filled in the order P_A(j), P_B(j), P_A(j+1) -- head A waits for
    P.V_B(j-1), head B for P.V_A(j), before writing it -- O per head, and the
    epilogue staging each head's output rows through that head's Q tile.
    cross_wait=False drops head B's wait for P.V_A(j) (to show the model
    notices when the shared P buffer is overwritten early)."""
    rng = random.Random(seed)
    B = {"q_full": Barrier(1), "mma_done": Barrier(1)}
    for s in range(STAGES):
        for n in ("k_full", "k_empty", "v_full", "v_empty"):
            B[f"{n}{s}"] = Barrier(1)
    for h in range(2):
        B[f"s_full{h}"] = Barrier(1)
        B[f"s_free{h}"] = Barrier(4)
        B[f"p_full{h}"] = Barrier(4)
        B[f"pv_done{h}"] = Barrier(1)
    smem = {"Q0": None, "Q1": None, "P": [None] * 4}
    for s in range(STAGES):
        smem[f"K{s}"] = smem[f"V{s}"] = None
    tmem = {"S0": [None] * 4, "S1": [None] * 4, "O0": set(), "O1": set()}
    tma, pipe = [], []

    def load(region, tile, bar):
        B[bar].expect_tx(1)
        tma.append((region, tile, bar))

    def producer():
        B["q_full"].expect_tx(2)  # one arrival expecting both Q tiles' bytes
        tma.append(("Q0", 0, "q_full"))
        tma.append(("Q1", 0, "q_full"))
        load("K0", 0, "k_full0")
        yield None
        for j in range(ntiles):
            if j + 1 < ntiles:
                t, st = j + 1, (j + 1) % STAGES
                if t >= STAGES:
                    yield lambda st=st, t=t: B[f"k_empty{st}"].test(((t // STAGES) - 1) & 1)
                load(f"K{st}", t, f"k_full{st}")
            st = j % STAGES
            if j >= STAGES:
                yield lambda st=st, j=j: B[f"v_empty{st}"].test(((j // STAGES) - 1) & 1)
            load(f"V{st}", j, f"v_full{st}")
            yield None

    def issue_qk(j):
        st = j % STAGES
        yield lambda: B[f"k_full{st}"].test((j // STAGES) & 1)
        for h in range(2):
            if j >= 1:
                yield lambda h=h: B[f"s_free{h}"].test((j - 1) & 1)
            pipe.append(("QK", h, j, st))
            pipe.append(("commit", f"s_full{h}"))
        pipe.append(("commit", f"k_empty{st}"))

    def issue_pv(j, h):
        yield lambda: B[f"p_full{h}"].test(j & 1)
        st = j % STAGES
        if h == 0:
            yield lambda: B[f"v_full{st}"].test((j // STAGES) & 1)
        pipe.append(("PV", h, j, st))
        pipe.append(("commit", f"pv_done{h}"))
        if h == 1:
            pipe.append(("commit", f"v_empty{st}"))

    def mma():
        yield None
        yield lambda: B["q_full"].test(0)
        yield from issue_qk(0)
        for j in range(ntiles):
            if j + 1 < ntiles:
                yield from issue_qk(j + 1)
            yield from issue_pv(j, 0)
            yield from issue_pv(j, 1)
        pipe.append(("commit", "mma_done"))
        yield lambda: B["mma_done"].test(0)

    def softmax(h, w):
        yield None
        for j in range(ntiles):
            yield lambda j=j: B[f"s_full{h}"].test(j & 1)
            if tmem[f"S{h}"][w] != ("S", j):
                raise Race(f"softmax {h}/{w} tile {j} read S lanes holding {tmem[f'S{h}'][w]}")
            B[f"s_free{h}"].arrive()
            yield None
            if h == 0 and j >= 1:
                yield lambda j=j: B["pv_done1"].test((j - 1) & 1)
            elif h == 1 and cross_wait:
                yield lambda j=j: B["pv_done0"].test(j & 1)
            smem["P"][w] = (h, j)
            if j >= 1 and rng.random() < 0.3 and set(range(j)) - tmem[f"O{h}"]:
                raise Race(f"softmax {h}/{w} rescaled O before P.V {sorted(set(range(j)) - tmem[f'O{h}'])}")
            B[f"p_full{h}"].arrive()
            yield None
        yield lambda: B[f"pv_done{h}"].test((ntiles - 1) & 1)
        if tmem[f"O{h}"] != set(range(ntiles)):
            raise Race(f"epilogue {h}/{w} read O with {sorted(tmem[f'O{h}'])}")
        smem[f"Q{h}"] = "staging"  # the epilogue stages output rows in Q_h

    actors = [producer(), mma()] + [softmax(h, w) for h in range(2) for w in range(4)]
    waiting = [None] * len(actors)
    done = [False] * len(actors)

    def step_pipe():
        op = pipe.pop(0)
        if op[0] == "QK":
            _, h, j, st = op
            if smem[f"Q{h}"] != 0 or smem[f"K{st}"] != j:
                raise Race(f"Q.K^T_{h}({j}) read Q={smem[f'Q{h}']} K{st}={smem[f'K{st}']}")
            tmem[f"S{h}"] = [("S", j)] * 4
        elif op[0] == "PV":
            _, h, j, st = op
            if smem["P"] != [(h, j)] * 4:
                raise Race(f"P.V_{h}({j}) read P holding {smem['P']}")
            if smem[f"V{st}"] != j:
                raise Race(f"P.V_{h}({j}) read V{st}={smem[f'V{st}']}")
            tmem[f"O{h}"].add(j)
        else:
            B[op[1]].arrive()

    for _ in range(400000):
        choices = [("actor", a) for a in range(len(actors))
                   if not done[a] and (waiting[a] is None or waiting[a]())]
        if pipe:
            choices.append(("pipe", None))
        if tma:
            choices.append(("tma", None))
        if not choices:
            if all(done):
                return
            raise Race(f"deadlock: waiting actors {[a for a in range(len(actors)) if not done[a]]}")
        kind, a = rng.choice(choices)
        if kind == "pipe":
            step_pipe()
        elif kind == "tma":
            region, tile, bar = tma.pop(rng.randrange(len(tma)))
            smem[region] = tile
            B[bar].complete_tx(1)
        else:
            try:
                waiting[a] = next(actors[a])
            except StopIteration:
                done[a] = True
    raise Race("no termination")


@pytest.mark.parametrize("ntiles", [1, 2, 3, 5, 8])
def test_pair_kernel_protocol_under_random_timing(ntiles):
    for seed in range(300):
        run_pair(ntiles, seed * 1000 + ntiles)


def test_pair_model_notices_an_early_p_overwrite():
    caught = []
    for seed in range(200):
        try:
            run_pair(4, seed, cross_wait=False)
        except Race as e:
            caught.append(str(e))
    assert any("read P holding" in c for c in caught), caught[:3]
