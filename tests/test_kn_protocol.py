"""Barrier protocol of the keys-in-lanes kernel (csrc/seg_kn.cu), checked on the CPU.

The kernel's roles are restated as coroutines over mbarriers with the
hardware's parity rule (``try_wait.parity(P)`` / ``test_wait.parity(P)``
succeed iff the count of completed phases is odd when P is 0, even when P is
1):

* scheduler -- decodes task k into slot k % 8 once ``task_empty`` shows the
  seven readers of task k - 8 (K producer, V producer, MMA issuer, four softmax
  warps) are done, publishes it on ``task_full``, gathers the Q^T rows of each
  task with tiles into buffer qi % QB once ``q_empty`` shows the last S of task
  qi - QB complete, and publishes a gather one task later -- or at once, before
  any wait that would block, and at the end;
* K and V producers -- copy each slot, release it, and stream the task's tiles
  through an S-stage ring (``*_full`` / ``*_empty``);
* MMA issuer -- one thread polling two cursors: S(g) up to three tiles ahead of
  P.V, each S once its Q^T (first tile of a task) and K tile are in, each P.V
  once P(g) and V(g) are; commits S_FULL / K_EMPTY / Q_EMPTY (a task's last S)
  and V_EMPTY / PV_DONE; the trailing cursor copies and releases the slots;
* softmax (the four warps as one role, four arrivals) -- per tile waits S(g),
  may wait for P.V(g-1) to rescale O, writes P(g) into buffer g % 3 and
  publishes it; a task's epilogue (reading its O^T buffer, by task parity) is
  deferred past the next task's first tile and waits for its last P.V; a task
  without tiles runs the pending epilogue first and is released at once.

This model found two stalls in lists holding long runs of tasks without tiles
(empty decode tails): the softmax deferred a pending epilogue -- and with it
the release of that task's slot -- past such tasks, and the issuer's trailing
cursor released their slots only while a P.V was outstanding; either way the
scheduler waited for a slot whose release waited for a task it could not
publish.  The kernel now runs the pending epilogue before a task without tiles
and settles the trailing slots (up to the lead) on every pass.

A random, speed-skewed scheduler interleaves the roles, lands copies in any
order and completes MMAs in issue order.  Every run must finish; every parity
wait or test must be evaluated while its barrier is at the awaited phase or one
past it; and no buffer (task slot, Q^T, K / V ring slot, S^T in TMEM, P^T,
O^T) may be rewritten while an earlier use still reads it.
"""
import random

import pytest

LOOK, TQ = 3, 8


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
    def __init__(self, ntiles, stages, qbufs, rng):
        self.tasks = ntiles              # tiles per task of this CTA's list (0: none)
        self.count = len(ntiles)
        self.S, self.QB, self.rng = stages, qbufs, rng
        mk = lambda name, n, count=1: [Bar(f"{name}{i}", count) for i in range(n)]
        self.k_full, self.k_empty = mk("K_FULL", stages), mk("K_EMPTY", stages)
        self.v_full, self.v_empty = mk("V_FULL", stages), mk("V_EMPTY", stages)
        self.s_full, self.p_full, self.pv_done = mk("S_FULL", LOOK), mk("P_FULL", LOOK, 4), mk("PV_DONE", LOOK)
        self.q_full, self.q_empty = mk("Q_FULL", qbufs), mk("Q_EMPTY", qbufs)
        self.task_full, self.task_empty = mk("TASK_FULL", TQ), mk("TASK_EMPTY", TQ, 7)
        self.slot = [None] * TQ          # task held by each slot
        self.qbuf = [None] * qbufs       # task-with-tiles index gathered into each Q^T buffer
        self.ring = {"K": [None] * stages, "V": [None] * stages}
        self.tma, self.pipe = [], []
        self.p_published = set()         # tiles whose P was published (S buffer read out)
        self.pv_complete, self.s_complete = set(), set()
        self.s_of_task, self.pv_of_task = {}, {}   # qi -> tiles
        self.epi_done = set()            # qi whose epilogue read its O^T buffer
        self.reading_q = [0] * qbufs     # S MMAs in the pipe reading each Q^T buffer
        self.reading = {"K": [0] * stages, "V": [0] * stages}

    # -- barrier rules ----------------------------------------------------------
    def ok(self, bar, phase):
        assert bar.done in (phase, phase + 1), f"{bar.name}: waiting for phase {phase} at {bar.done}"
        return bar.done % 2 != phase % 2

    def read_slot(self, k):
        assert self.slot[k % TQ] == k, f"slot {k % TQ} read for task {k} holds {self.slot[k % TQ]}"
        return self.tasks[k]

    # -- scheduler ----------------------------------------------------------------
    def scheduler(self):
        qi, pending = 0, None

        def flush():
            nonlocal pending
            if pending is not None:
                self.q_full[pending % self.QB].arrive()
                pending = None

        for k in range(self.count):
            if k >= TQ:
                bar, ph = self.task_empty[k % TQ], k // TQ - 1
                if not self.ok(bar, ph):
                    flush()
                    yield ("wait", bar, ph)
            self.slot[k % TQ] = k
            self.task_full[k % TQ].arrive()
            yield ("step",)
            if self.tasks[k] == 0:
                continue
            qb = qi % self.QB
            if qi >= self.QB:
                bar, ph = self.q_empty[qb], qi // self.QB - 1
                if not self.ok(bar, ph):
                    flush()
                    yield ("wait", bar, ph)
                prev = qi - self.QB
                assert self.reading_q[qb] == 0 and self.s_of_task.get(prev, set()) <= self.s_complete, \
                    "Q^T buffer regathered while an S reads it"
            self.qbuf[qb] = qi
            if qi == 0:
                self.q_full[qb].arrive()
            else:
                flush()
                pending = qi
            qi += 1
            yield ("step",)
        flush()

    # -- producers ------------------------------------------------------------------
    def producer(self, which):
        full, empty = (self.k_full, self.k_empty) if which == "K" else (self.v_full, self.v_empty)
        g = 0
        for k in range(self.count):
            yield ("wait", self.task_full[k % TQ], k // TQ)
            n = self.read_slot(k)
            self.task_empty[k % TQ].arrive()
            for _ in range(n):
                st = g % self.S
                if g >= self.S:
                    yield ("wait", empty[st], g // self.S - 1)
                assert self.reading[which][st] == 0, f"{which} slot refilled while an MMA reads it"
                self.tma.append((full[st], which, st, g))
                g += 1
                yield ("step",)
        for q in range(max(0, g - self.S), g):
            yield ("wait", full[q % self.S], q // self.S)

    # -- MMA issuer ------------------------------------------------------------------
    def mma(self, kind, g, qi, reads):
        for ring, st, tile in reads:
            if ring == "Q":
                assert self.qbuf[st] == tile, f"S reads Q^T of task {tile} from a buffer holding {self.qbuf[st]}"
                self.reading_q[st] += 1
            else:
                assert self.ring[ring][st] == tile, f"MMA reads {ring}({tile}) from a slot holding {self.ring[ring][st]}"
                self.reading[ring][st] += 1
        self.pipe.append(("mma", (kind, g, qi, reads)))

    def commit(self, bar):
        self.pipe.append(("commit", bar))

    def issuer(self):
        S, QB = self.S, self.QB
        sc = dict(k=0, j=0, g=0, qi=0, t=None, loaded=False)
        pc = dict(k=0, j=0, g=0, qi=0, t=None, loaded=False)

        def lead_ready():
            while sc["k"] < self.count:
                if not sc["loaded"]:
                    if not self.ok(self.task_full[sc["k"] % TQ], sc["k"] // TQ):
                        return ("wait", self.task_full[sc["k"] % TQ], sc["k"] // TQ)
                    sc["t"], sc["loaded"] = self.read_slot(sc["k"]), True
                if sc["t"] > 0:
                    return True
                sc["k"] += 1
                sc["loaded"] = False
            return False

        def trail_settle():   # never past the lead
            while pc["k"] < self.count and not pc["loaded"] and \
                    (pc["k"] < sc["k"] or (pc["k"] == sc["k"] and sc["loaded"])):
                pc["t"] = self.read_slot(pc["k"])
                self.task_empty[pc["k"] % TQ].arrive()
                if pc["t"] > 0:
                    pc["loaded"] = True
                    break
                pc["k"] += 1

        while True:
            did, blockers = False, []
            if not pc["loaded"]:
                trail_settle()
            if pc["g"] < sc["g"]:
                if not pc["loaded"]:
                    trail_settle()
                g, st = pc["g"], pc["g"] % S
                a = self.ok(self.p_full[g % LOOK], g // LOOK)
                b = self.ok(self.v_full[st], g // S)
                if a and b:
                    assert pc["j"] > 0 or pc["qi"] < 2 or pc["qi"] - 2 in self.epi_done, \
                        "P.V overwrites an O^T buffer before its epilogue read it"
                    self.mma("pv", g, pc["qi"], [("V", st, g)])
                    self.pv_of_task.setdefault(pc["qi"], set()).add(g)
                    self.commit(self.v_empty[st])
                    self.commit(self.pv_done[g % LOOK])
                    pc["g"] += 1
                    pc["j"] += 1
                    if pc["j"] >= pc["t"]:
                        pc["j"], pc["k"], pc["qi"], pc["loaded"] = 0, pc["k"] + 1, pc["qi"] + 1, False
                    did = True
                else:
                    blockers += [("wait", self.p_full[g % LOOK], g // LOOK), ("wait", self.v_full[st], g // S)]
            if sc["g"] - pc["g"] < LOOK:
                r = lead_ready()
                if r is True:
                    g, st, qb = sc["g"], sc["g"] % S, sc["qi"] % QB
                    qok = sc["j"] != 0 or self.ok(self.q_full[qb], sc["qi"] // QB)
                    kok = self.ok(self.k_full[st], g // S)
                    if qok and kok:
                        assert g < LOOK or g - LOOK in self.p_published, "S overwrites an S^T buffer not yet read"
                        self.mma("s", g, sc["qi"], [("K", st, g), ("Q", qb, sc["qi"])])
                        self.s_of_task.setdefault(sc["qi"], set()).add(g)
                        self.commit(self.s_full[g % LOOK])
                        self.commit(self.k_empty[st])
                        if sc["j"] == sc["t"] - 1:
                            self.commit(self.q_empty[qb])
                        sc["g"] += 1
                        sc["j"] += 1
                        if sc["j"] >= sc["t"]:
                            sc["j"], sc["k"], sc["qi"], sc["loaded"] = 0, sc["k"] + 1, sc["qi"] + 1, False
                        did = True
                    else:
                        if sc["j"] == 0:
                            blockers.append(("wait", self.q_full[qb], sc["qi"] // QB))
                        blockers.append(("wait", self.k_full[st], g // S))
                elif r:
                    blockers.append(r)
            if sc["k"] >= self.count and pc["g"] == sc["g"]:
                break
            # the kernel polls: any pass may also settle trailing slots
            blockers.append(("until", lambda: not pc["loaded"] and pc["k"] < self.count and
                             (pc["k"] < sc["k"] or (pc["k"] == sc["k"] and sc["loaded"]))))
            yield ("step",) if did else ("any", blockers)
        trail_settle()
        total = pc["g"]
        for q in range(max(0, total - S), total):
            yield ("wait", self.k_empty[q % S], q // S)
            yield ("wait", self.v_empty[q % S], q // S)

    # -- softmax warps ----------------------------------------------------------------
    def release(self, k):
        for _ in range(4):
            self.task_empty[k % TQ].arrive()

    def epilogue(self, k, g_last, qi):
        yield ("wait", self.pv_done[g_last % LOOK], g_last // LOOK)
        self.read_slot(k)
        assert self.pv_of_task[qi] <= self.pv_complete, "epilogue before its task's last P.V"
        assert qi + 2 not in self.pv_of_task, "O^T buffer rewritten before its epilogue"
        self.epi_done.add(qi)
        self.release(k)

    def softmax(self):
        g, qi, pend = 0, 0, None
        for k in range(self.count):
            yield ("wait", self.task_full[k % TQ], k // TQ)
            n = self.read_slot(k)
            if n == 0:
                if pend is not None:     # nothing to overlap it with: the pending epilogue runs now
                    yield from self.epilogue(*pend)
                    pend = None
                self.release(k)
                continue
            for j in range(n):
                yield ("wait", self.s_full[g % LOOK], g // LOOK)
                if j > 0 and self.rng.random() < 0.3:      # a row maximum grew: rescale O after P.V(g-1)
                    yield ("wait", self.pv_done[(g - 1) % LOOK], (g - 1) // LOOK)
                assert g < LOOK or g - LOOK in self.pv_complete, "P overwrites a P^T buffer a P.V still reads"
                self.p_published.add(g)
                for _ in range(4):
                    self.p_full[g % LOOK].arrive()
                if j == 0 and pend is not None:
                    yield from self.epilogue(*pend)
                    pend = None
                g += 1
                yield ("step",)
            pend = (k, g - 1, qi)
            qi += 1
        if pend is not None:
            yield from self.epilogue(*pend)

    # -- scheduler of the model ------------------------------------------------------
    def ready(self, w):
        if w[0] == "step":
            return True
        if w[0] == "wait":
            return self.ok(w[1], w[2])
        if w[0] == "until":
            return w[1]()
        return any(self.ready(x) for x in w[1])

    def run(self):
        agents = [self.scheduler(), self.producer("K"), self.producer("V"), self.issuer(), self.softmax()]
        waits = [("step",)] * len(agents)
        live = list(range(len(agents)))
        speed = {("agent", i): self.rng.choice([0.02, 1.0, 1.0, 8.0]) for i in range(len(agents))}
        speed[("tma", None)] = self.rng.choice([0.05, 1.0, 8.0])
        speed[("pipe", None)] = self.rng.choice([0.05, 1.0, 8.0])
        for _ in range(200000):
            ready = [("agent", i) for i in live if self.ready(waits[i])]
            if self.tma:
                ready.append(("tma", None))
            if self.pipe:
                ready.append(("pipe", None))
            if not ready:
                assert not live, f"deadlock: {[(i, waits[i]) for i in live]}"
                return
            kind, i = self.rng.choices(ready, weights=[speed[r] for r in ready])[0]
            if kind == "agent":
                try:
                    waits[i] = next(agents[i])
                except StopIteration:
                    live.remove(i)
            elif kind == "tma":
                bar, ring, st, g = self.tma.pop(self.rng.randrange(len(self.tma)))
                self.ring[ring][st] = g
                bar.arrive()
            else:
                op, arg = self.pipe.pop(0)
                if op == "commit":
                    arg.arrive()
                    continue
                kind2, g, qi, reads = arg
                for ring, st, _ in reads:
                    if ring == "Q":
                        self.reading_q[st] -= 1
                    else:
                        self.reading[ring][st] -= 1
                (self.s_complete if kind2 == "s" else self.pv_complete).add(g)
        raise AssertionError("no progress bound reached")


@pytest.mark.parametrize("stages", [1, 2, 3])
@pytest.mark.parametrize("qbufs", [2, 4])
@pytest.mark.parametrize("shape", ["ones", "mixed", "long", "sparse"])
def test_keys_in_lanes_barrier_protocol(stages, qbufs, shape):
    for seed in range(120):
        rng = random.Random(seed * 7919 + stages * 31 + qbufs)
        count = rng.randint(1, 20)
        if shape == "ones":
            tasks = [1] * count
        elif shape == "mixed":
            tasks = [rng.choice([0, 1, 1, 2, 3]) for _ in range(count)]
        elif shape == "long":
            tasks = [rng.randint(1, 6) for _ in range(count)]
        else:   # runs of tasks without tiles longer than the task ring
            tasks = [rng.choice([0] * 6 + [1, 2]) for _ in range(count + 10)]
        cta = Cta(tasks, stages, qbufs, rng)
        cta.run()
        assert len(cta.epi_done) == sum(1 for t in tasks if t > 0)


def test_large_decode_batch_has_long_runs_of_tasks_without_tiles():
    """The stall the model found is reachable: a cached decode plan for 1200 requests puts, in some
    keys-in-lanes CTA's list, 8 or more growing tails in a row after a task with tiles -- at the step
    where the tails are still empty every one of them is a task without tiles."""
    import numpy as np
    from tree_attention import CostModel, KVTree, kernels, schedule
    from tree_attention.schedule import Job, physical_jobs
    nreq, steps = 1200, 2
    tree = KVTree.synthetic([-1] + [0] * nreq, [512] + [16] * nreq, list(range(1, nreq + 1)))
    plan = schedule(tree, 32, 8, 128, "cube", CostModel.b200())
    prefix = tree.storage_tokens
    tails = [Job((r,), tuple(range(prefix + r * steps, prefix + (r + 1) * steps))) for r in range(nreq)]
    jobs = physical_jobs(plan.jobs + tails)
    jobs.sort(key=lambda job: len(job.requests) * 4 > 16)
    meta = kernels.build_metadata(jobs, nreq, 4, True, heads=8, sms=148, no_split_from=prefix)
    offsets, tasks, segs = (np.asarray(meta[key]) for key in ("kn_offsets", "kn_tasks", "kn_segs"))
    growing = ((segs[:, 7] >> 30) & 1).astype(bool)
    empty = np.array([growing[t[0]:t[0] + t[1]].all() for t in tasks])
    longest = 0
    for c in range(len(offsets) - 1):
        run, seen_tiles = 0, False
        for e in empty[offsets[c]:offsets[c + 1]]:
            run = run + 1 if (e and seen_tiles) else 0
            seen_tiles |= not e
            longest = max(longest, run)
    assert longest >= 8
