"""Discrete-event models of the prefill kernel's barrier protocol
(``kp3_kernel`` in ``halo_b200/csrc/prefill.cu``), for the CPU tests.

Roles: one producer streams K/V tiles through an ST-stage ring (full
barriers: one arrival + the copy's bytes; empty barriers: one arrival per
query tile, the producer arriving for a tile that sits the K/V tile out);
MMA issuers (QK into score buffers, P V into O; ``tcgen05.commit`` arrivals
complete in issue order per issuing thread) and per query tile X a softmax
group (waits S, writes P).  Query tile A sees a prefix of each segment's
K/V tiles; tile B sees all of them.

Barriers count completed phases.  A wait for phase n by parity succeeds when
n has completed; it is an error (in hardware: a stall or an early return) if
the barrier is then at neither n nor n + 1 completed phases -- in particular
a probe of phase n while phase n - 1 is still open reads as complete.

``simulate_kernel`` is the kernel: ONE issuing thread for both query tiles
that polls and issues whichever of the four next steps (QK / P V of A / B)
has its inputs ready, one 128-key score buffer per tile (QK_X(j+1) after
PV_X(j) completed), tile B's first QK after tile A's first P V when both
start on the walk's first K/V tile.  K and V landings are observed in walk
order (a landed prefix per ring), so a tile that sits K/V tiles out never
probes a ring stage whose previous use has not been seen to land.

``simulate`` models the alternative of one issuing thread per query tile
with score buffers ``NB`` deep and ``SPT`` score tiles per K/V tile:
``issuer="blocking"`` (QK NB score tiles ahead of P V, each step waiting for
its inputs, waiting on the full barriers of tiles it sits out) stalls when
tile A sits out two K/V tiles in a row; ``issuer="polling"`` does not."""
from __future__ import annotations

import random


class Stall(Exception):
    """The protocol deadlocked or a parity wait aliased."""


class _Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.tx, self.phase = name, count, count, 0, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0, f"{self.name}: too many arrivals"
        self._maybe()

    def expect_tx(self):
        self.tx += 1
        self.arrive()

    def land(self):
        self.tx -= 1
        self._maybe()

    def _maybe(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count


def _done(bar, n):
    """A parity probe for the completion of phase ``n`` (hardware: true iff
    the current phase's parity differs from n's).  With c phases completed
    it answers correctly only for c in {n, n + 1}: c = n - 1 would read as
    done, c >= n + 2 as done or not by parity alone."""
    c = bar.phase
    if c >= n + 2 or c == n - 1:
        raise Stall(f"aliased wait: {bar.name} probes phase {n}, {c} completed")
    return c == n + 1


def _wait(bar, n):
    while not _done(bar, n):
        yield


def tiles_of(segs):
    """segs: [(tiles B sees, tiles A sees)] -> [A takes tile?] in walk order."""
    return [t < n_a for n_u, n_a in segs for t in range(n_u)]


def simulate(segs, ST, NB=2, SPT=2, issuer="blocking", seed=0, max_steps=100000):
    """Run one random schedule of a CTA with both query tiles; raise Stall on
    a deadlock or an aliased wait."""
    rng = random.Random(seed)
    takes_a = tiles_of(segs)
    n = len(takes_a)
    bars = []

    def bar(name, count):
        bars.append(_Bar(name, count))
        return bars[-1]
    q_full = bar("q_full", 1)
    k_full = [bar(f"k_full{i}", 1) for i in range(ST)]
    v_full = [bar(f"v_full{i}", 1) for i in range(ST)]
    k_empty = [bar(f"k_empty{i}", 2) for i in range(ST)]
    v_empty = [bar(f"v_empty{i}", 2) for i in range(ST)]
    s_full = [[bar(f"s_full{x}{b}", 1) for b in range(2)] for x in range(2)]
    p_full = [[bar(f"p_full{x}{b}", 1) for b in range(2)] for x in range(2)]
    pv_done = [[bar(f"pv_done{x}{b}", 1) for b in range(2)] for x in range(2)]
    now, seq, events = [0], [0], []
    last_commit = [0, 0]

    def later(delay, fn):
        seq[0] += 1
        events.append((now[0] + delay, seq[0], fn))

    def commit(x, b, k=1):
        t = max(now[0] + rng.randint(1, 6), last_commit[x])
        last_commit[x] = t
        seq[0] += 1
        events.append((t, seq[0], lambda: b.arrive(k)))

    def producer():
        q_full.expect_tx()
        later(rng.randint(1, 5), q_full.land)
        for g, ta in enumerate(takes_a):
            st, use = g % ST, g // ST
            absent = 0 if ta else 1
            if use > 0:
                yield from _wait(k_empty[st], use - 1)
            k_full[st].expect_tx()
            later(rng.randint(1, 8), k_full[st].land)
            if absent:
                k_empty[st].arrive(absent)
            if use > 0:
                yield from _wait(v_empty[st], use - 1)
            v_full[st].expect_tx()
            later(rng.randint(1, 8), v_full[st].land)
            if absent:
                v_empty[st].arrive(absent)

    def mma_issuer(x):
        takes = (lambda g: True) if x else (lambda g: takes_a[g])
        c = dict(q=0, p=0, hq=0, hp=0, jq=0, jp=0)
        yield from _wait(q_full, 0)
        if x == 1 and segs[0][1] > 0:
            yield from _wait(p_full[0][0], 0)      # tile B starts after A's first P

        def do_qk():
            g = c["q"]
            st, j = g % ST, c["jq"]
            commit(x, s_full[x][j % NB])
            c["jq"] += 1
            if c["hq"] == SPT - 1:
                commit(x, k_empty[st])
                c["q"] += 1
                c["hq"] = 0
            else:
                c["hq"] += 1

        def do_pv():
            g = c["p"]
            st, j = g % ST, c["jp"]
            commit(x, pv_done[x][j % NB])
            c["jp"] += 1
            if c["hp"] == SPT - 1:
                commit(x, v_empty[st])
                c["p"] += 1
                c["hp"] = 0
            else:
                c["hp"] += 1

        if issuer == "polling":
            while True:
                while c["q"] < n and not takes(c["q"]):
                    c["q"] += 1
                while c["p"] < n and not takes(c["p"]):
                    c["p"] += 1
                if c["q"] >= n and c["jp"] == c["jq"]:
                    return
                did = False
                if c["q"] < n:
                    g, j = c["q"], c["jq"]
                    if (c["hq"] > 0 or _done(k_full[g % ST], g // ST)) and \
                            (j < NB or _done(pv_done[x][j % NB], (j - NB) // NB)):
                        do_qk()
                        did = True
                if c["jp"] < c["jq"]:
                    g, j = c["p"], c["jp"]
                    if (c["hp"] > 0 or _done(v_full[g % ST], g // ST)) and \
                            _done(p_full[x][j % NB], j // NB):
                        do_pv()
                        did = True
                if not did:
                    yield
            return

        def qk_step():
            while c["q"] < n and not takes(c["q"]):
                g = c["q"]
                yield from _wait(k_full[g % ST], g // ST)
                c["q"] += 1
            if c["q"] >= n:
                return 0
            g, j = c["q"], c["jq"]
            if c["hq"] == 0:
                yield from _wait(k_full[g % ST], g // ST)
            if j >= NB:
                yield from _wait(pv_done[x][j % NB], (j - NB) // NB)
            do_qk()
            return 1

        def pv_step():
            while not takes(c["p"]):
                g = c["p"]
                yield from _wait(v_full[g % ST], g // ST)
                c["p"] += 1
            g, j = c["p"], c["jp"]
            if c["hp"] == 0:
                yield from _wait(v_full[g % ST], g // ST)
            yield from _wait(p_full[x][j % NB], j // NB)
            do_pv()

        rq = yield from qk_step()
        if NB == 2 and rq > 0:
            rq = yield from qk_step()
        while c["jp"] < c["jq"]:
            yield from pv_step()
            if rq > 0:
                rq = yield from qk_step()

    def softmax(x):
        count = n if x else sum(takes_a)
        j = 0
        for _ in range(count * SPT):
            yield from _wait(s_full[x][j % NB], j // NB)
            if j > 0 and rng.random() < 0.3:       # O rescale
                yield from _wait(pv_done[x][(j - 1) % NB], (j - 1) // NB)
            p_full[x][j % NB].arrive()
            j += 1
        if j > 0:
            yield from _wait(pv_done[x][(j - 1) % NB], (j - 1) // NB)

    live = {"producer": producer(), "issuerA": mma_issuer(0), "issuerB": mma_issuer(1),
            "softmaxA": softmax(0), "softmaxB": softmax(1)}
    for step in range(max_steps):
        if not live and not events:
            return
        for name in rng.sample(list(live), len(live)):
            try:
                next(live[name])
            except StopIteration:
                del live[name]
        if events and (rng.random() < 0.5 or not live):
            events.sort()
            t, _, fn = events.pop(0)
            now[0] = max(now[0], t)
            fn()
    raise Stall("deadlock: " + ", ".join(sorted(live)) + "; " +
                ", ".join(f"{b.name}={b.phase}" for b in bars))


def max_sit_out_run(segs):
    """Longest run of consecutive K/V tiles that query tile A sits out."""
    run = best = 0
    for takes in tiles_of(segs):
        run = 0 if takes else run + 1
        best = max(best, run)
    return best


def simulate_kernel(segs, ST, seed=0, has_b=True, max_steps=200000):
    """One random schedule of ``kp3_kernel``'s protocol; raise Stall on a
    deadlock or an aliased wait.  ``segs``: [(tiles B sees, tiles A sees)];
    with ``has_b=False`` only tile A exists (its tiles form the walk)."""
    rng = random.Random(seed)
    if not has_b:
        segs = [(n_a, n_a) for _n_u, n_a in segs]
    takes_a = tiles_of(segs)
    n = len(takes_a)
    n_x = [sum(takes_a), n if has_b else 0]
    bars = []

    def bar(name, count):
        bars.append(_Bar(name, count))
        return bars[-1]
    q_full = bar("q_full", 1)
    k_full = [bar(f"k_full{i}", 1) for i in range(ST)]
    v_full = [bar(f"v_full{i}", 1) for i in range(ST)]
    k_empty = [bar(f"k_empty{i}", 2) for i in range(ST)]
    v_empty = [bar(f"v_empty{i}", 2) for i in range(ST)]
    s_full = [bar(f"s_full{x}", 1) for x in range(2)]
    p_full = [bar(f"p_full{x}", 1) for x in range(2)]
    pv_done = [bar(f"pv_done{x}", 1) for x in range(2)]
    now, seq, events = [0], [0], []
    last_commit = [0]

    def later(delay, fn):
        seq[0] += 1
        events.append((now[0] + delay, seq[0], fn))

    def commit(b):
        # one issuing thread: its commits complete in issue order
        t = max(now[0] + rng.randint(1, 6), last_commit[0])
        last_commit[0] = t
        seq[0] += 1
        events.append((t, seq[0], b.arrive))

    def producer():
        if n == 0:
            return
        q_full.expect_tx()
        later(rng.randint(1, 5), q_full.land)
        for g, ta in enumerate(takes_a):
            st, use = g % ST, g // ST
            absent = (0 if ta else 1) + (0 if has_b else 1)
            if use > 0:
                yield from _wait(k_empty[st], use - 1)
            k_full[st].expect_tx()
            later(rng.randint(1, 8), k_full[st].land)
            if absent:
                k_empty[st].arrive(absent)
            if use > 0:
                yield from _wait(v_empty[st], use - 1)
            v_full[st].expect_tx()
            later(rng.randint(1, 8), v_full[st].land)
            if absent:
                v_empty[st].arrive(absent)

    def issuer():
        if n == 0:
            return
        takes = [lambda g: takes_a[g], lambda g: has_b]
        qc, pc = [0, 0], [0, 0]
        jq, jp = [0, 0], [0, 0]

        def seek(c, x):
            while c < n and not takes[x](c):
                c += 1
            return c
        for x in range(2):
            qc[x] = seek(0, x)
            pc[x] = seek(0, x)
        # landed prefixes: K/V tiles below kpre / vpre are known to have
        # landed; the next one is probed in walk order, so every probe of a
        # stage follows the observed landing of its previous use
        kpre = vpre = 0
        yield from _wait(q_full, 0)
        while True:
            did = False
            while kpre < n and _done(k_full[kpre % ST], kpre // ST):
                kpre += 1
            while vpre < n and _done(v_full[vpre % ST], vpre // ST):
                vpre += 1
            for x in range(2):
                if jp[x] < jq[x]:
                    g = pc[x]
                    if g < vpre and _done(p_full[x], jp[x]):
                        commit(pv_done[x])
                        commit(v_empty[g % ST])
                        jp[x] += 1
                        pc[x] = seek(g + 1, x)
                        did = True
                if jq[x] < n_x[x] and jq[x] == jp[x]:
                    g = qc[x]
                    if g < kpre and (jq[x] == 0 or _done(pv_done[x], jq[x] - 1)):
                        commit(s_full[x])
                        commit(k_empty[g % ST])
                        jq[x] += 1
                        qc[x] = seek(g + 1, x)
                        did = True
            if jp[0] >= n_x[0] and jp[1] >= n_x[1]:
                return
            if not did:
                yield

    def softmax(x):
        for j in range(n_x[x]):
            yield from _wait(s_full[x], j)
            p_full[x].arrive()
        if n_x[x] > 0:
            yield from _wait(pv_done[x], n_x[x] - 1)

    live = {"producer": producer(), "issuer": issuer(), "softmaxA": softmax(0),
            "softmaxB": softmax(1)}
    for _step in range(max_steps):
        if not live and not events:
            # every barrier of the ring ends balanced: each stage's empty
            # phases match the loads that used it
            return
        for name in rng.sample(list(live), len(live)):
            try:
                next(live[name])
            except StopIteration:
                del live[name]
        if events and (rng.random() < 0.5 or not live):
            events.sort()
            t, _, fn = events.pop(0)
            now[0] = max(now[0], t)
            fn()
    raise Stall("deadlock: " + ", ".join(sorted(live)) + "; " +
                ", ".join(f"{b.name}={b.phase}" for b in bars))
