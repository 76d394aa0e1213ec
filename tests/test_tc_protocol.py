"""Barrier protocol of the query-tile kernel (csrc/seg_tc.cu), checked on the CPU.

The kernel's roles -- K producer, V producer (with its start-up wait for the
first K tiles), the MMA issuer (V(j)/K(j+1) waits ahead of tile A's P(j)), the
two softmax warpgroups and their epilogues -- are restated here as coroutines
over mbarriers with the hardware's parity-wait rule: ``try_wait.parity(P)``
succeeds iff the number of completed phases is odd when P is 0 and even when
P is 1.  A random scheduler interleaves the roles, lands TMA copies in any
order and completes MMAs in issue order (one issuing thread).  Every run must
finish, and every parity wait must be evaluated while its barrier is at the
phase it waits for or one past it (a waiter one phase early would pass
wrongly, two phases late would never pass).  The epilogue's staging into a
ring must find every MMA that reads that ring complete, and an MMA must never
read a ring slot whose load has not landed or that was refilled since.
"""
import random

import pytest


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0, self.name
        if self.pending == 0:
            self.done += 1
            self.pending = self.count


class Cta:
    """One CTA of the kernel: `ntiles` K/V tiles, `ntile` query tiles (1 or 2),
    a partial last tile (`tail`) or not, queries by TMA (`tma_q`) or by the
    softmax threads."""

    def __init__(self, ntiles, ntile, tail, tma_q, rng):
        self.n, self.ntile, self.tail, self.tma_q, self.rng = ntiles, ntile, tail, tma_q, rng
        b = lambda name, count=1: Bar(name, count)
        self.k_full = [b("K_FULL0"), b("K_FULL1")]
        self.k_empty = [b("K_EMPTY0"), b("K_EMPTY1")]
        self.v_full = [b("V_FULL0"), b("V_FULL1")]
        self.v_empty = [b("V_EMPTY0"), b("V_EMPTY1")]
        self.s_full = [b("S_FULL0"), b("S_FULL1")]
        self.p_full = [b("P_FULL0", 4), b("P_FULL1", 4)]
        self.pv_done = [b("PV_DONE0"), b("PV_DONE1")]
        self.q_full = [b("Q_FULL0", 1 if tma_q else 4), b("Q_FULL1", 1 if tma_q else 4)]
        self.v_tail = b("V_TAIL")
        self.tma = []            # in-flight loads: (barrier, ring, slot, tile)
        self.pipe = []           # issued MMAs in order: ("mma", reads) or ("commit", barrier)
        self.ring = {"K": [None, None], "V": [None, None]}   # tile landed in each slot
        self.reading = {"K": [0, 0], "V": [0, 0]}            # MMAs in the pipe reading each slot
        self.v_zeroed = False

    # -- wait conditions (evaluated by the scheduler) --------------------------
    def parity_ok(self, bar, phase):
        assert bar.done in (phase, phase + 1), f"{bar.name}: waiting for phase {phase} at {bar.done}"
        return bar.done % 2 != phase % 2

    # -- roles ------------------------------------------------------------------
    def k_producer(self):
        if self.tma_q:
            for t in range(self.ntile):
                self.tma.append((self.q_full[t], None, None, None))
        for j in range(self.n):
            st = j % 2
            if j >= 2:
                yield ("wait", self.k_empty[st], j // 2 - 1)
            if j == 1:
                yield ("wait", self.q_full[0], 0)
            assert self.reading["K"][st] == 0, "K slot refilled while an MMA reads it"
            self.tma.append((self.k_full[st], "K", st, j))
            yield ("step",)

    def v_producer(self):
        for j in range(self.n):
            st = j % 2
            if j >= 2:
                yield ("wait", self.v_empty[st], j // 2 - 1)
            if j < 2:   # K(j) landed, or consumed already (the kernel's k_landed)
                yield ("until", lambda j=j: self.k_full[j].done % 2 == 1 or self.k_empty[j].done % 2 == 1)
            assert self.reading["V"][st] == 0, "V slot refilled while an MMA reads it"
            self.tma.append((self.v_full[st], "V", st, j))
            yield ("step",)
        if self.tail:
            last = self.n - 1
            yield ("wait", self.v_full[last % 2], last // 2)
            self.v_zeroed = True
            self.v_tail.arrive()

    def mma(self, ring, slot, tile):
        assert self.ring[ring][slot] == tile, f"MMA reads {ring}({tile}) from a slot holding {self.ring[ring][slot]}"
        self.reading[ring][slot] += 1
        self.pipe.append(("mma", (ring, slot)))

    def commit(self, bar):
        self.pipe.append(("commit", bar))

    def issuer(self):
        n = self.n
        yield ("wait", self.q_full[0], 0)
        yield ("wait", self.k_full[0], 0)
        self.mma("K", 0, 0)
        self.commit(self.s_full[0])
        if self.ntile == 2:
            yield ("wait", self.q_full[1], 0)
            self.mma("K", 0, 0)
            self.commit(self.s_full[1])
        self.commit(self.k_empty[0])
        for j in range(n):
            more = j + 1 < n
            zeroed = self.tail and j == n - 1
            if zeroed:
                yield ("wait", self.v_tail, 0)
                assert self.v_zeroed, "the last V tile is read before its rows past the segment are zeroed"
            else:
                yield ("wait", self.v_full[j % 2], j // 2)
            if more:
                yield ("wait", self.k_full[(j + 1) % 2], (j + 1) // 2)
            for t in range(self.ntile):
                yield ("wait", self.p_full[t], j)
                self.mma("V", j % 2, j)
                if j == n - 1:
                    self.commit(self.pv_done[t])
                if t == self.ntile - 1:
                    self.commit(self.v_empty[j % 2])
                if more:
                    self.mma("K", (j + 1) % 2, j + 1)
                    self.commit(self.s_full[t])
                    if t == self.ntile - 1:
                        self.commit(self.k_empty[(j + 1) % 2])
                yield ("step",)
        for j in range(max(0, n - 2), n):
            yield ("wait", self.k_empty[j % 2], j // 2)
        for j in range(max(0, n - 2), n):
            yield ("wait", self.v_empty[j % 2], j // 2)

    def softmax(self, t):
        if not self.tma_q:
            for _ in range(4):
                self.q_full[t].arrive()
        for j in range(self.n):
            yield ("wait", self.s_full[t], j)
            for _ in range(4):
                self.p_full[t].arrive()
            yield ("step",)
        yield ("wait", self.pv_done[t], 0)
        # staging into the K ring (tile A) or the V ring (tile B)
        ring = "K" if t == 0 else "V"
        assert self.reading[ring] == [0, 0], f"epilogue of tile {t} stages into the {ring} ring while MMAs read it"
        self.staged = getattr(self, "staged", 0) + 1

    # -- scheduler --------------------------------------------------------------
    def run(self):
        agents = [self.k_producer(), self.v_producer(), self.issuer()] + [self.softmax(t) for t in range(self.ntile)]
        waits = [("step",)] * len(agents)
        live = list(range(len(agents)))
        # per-run speeds: a slow role or slow copies make the skewed schedules likely
        speed = {("agent", i): self.rng.choice([0.02, 1.0, 1.0, 8.0]) for i in range(len(agents))}
        speed[("tma", None)] = self.rng.choice([0.05, 1.0, 8.0])
        speed[("pipe", None)] = self.rng.choice([0.05, 1.0, 8.0])
        for _ in range(100000):
            ready = []
            for i in live:
                w = waits[i]
                if w[0] == "step" or (w[0] == "wait" and self.parity_ok(w[1], w[2])) or (w[0] == "until" and w[1]()):
                    ready.append(("agent", i))
            if self.tma:
                ready.append(("tma", None))
            if self.pipe:
                ready.append(("pipe", None))
            if not ready:
                assert not live, f"deadlock: {[waits[i] for i in live]}"
                return
            kind, i = self.rng.choices(ready, weights=[speed[r] for r in ready])[0]
            if kind == "agent":
                try:
                    waits[i] = next(agents[i])
                except StopIteration:
                    live.remove(i)
            elif kind == "tma":
                bar, ring, slot, tile = self.tma.pop(self.rng.randrange(len(self.tma)))
                if ring is not None:
                    self.ring[ring][slot] = tile
                bar.arrive()
            else:   # the oldest MMA or commit completes (one issuing thread: in order)
                op, arg = self.pipe.pop(0)
                if op == "mma":
                    self.reading[arg[0]][arg[1]] -= 1
                else:
                    arg.arrive()
        raise AssertionError("no progress bound reached")


@pytest.mark.parametrize("ntiles", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("ntile", [1, 2])
@pytest.mark.parametrize("tail", [False, True])
@pytest.mark.parametrize("tma_q", [False, True])
def test_query_tile_barrier_protocol(ntiles, ntile, tail, tma_q):
    for seed in range(150):
        cta = Cta(ntiles, ntile, tail, tma_q, random.Random(seed * 1000 + ntiles))
        cta.run()
        assert cta.staged == ntile


def test_protocol_model_catches_a_late_waiter():
    """The parity rule of the model flags a waiter that falls two phases behind."""
    cta = Cta(2, 1, False, True, random.Random(0))
    bar = cta.k_full[0]
    bar.arrive()
    bar.arrive()
    with pytest.raises(AssertionError, match="waiting for phase 0 at 2"):
        cta.parity_ok(bar, 0)
