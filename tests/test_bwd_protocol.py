"""Model check of the backward main kernel's barrier protocol (csrc/swa_backward.cu,
`lca_bwd_main`), on the CPU.

Each role of one persistent CTA is restated as a generator that follows the kernel's loops
and waits: the S/dP issuer, the accumulate issuer, the producer (TMA ring, outer-tile
buffers, the key-major kernel's LSE/D staging) and the P/dS warps, which form two groups
taking alternate inner tiles (tile g to group g % 2).  Barriers are modelled as mbarriers:
an arrival count and a transaction count per phase, and waits by phase parity.  The
asynchronous work is modelled too:
- MMAs run in issue order per issuing thread, and a commit arrives once everything the
  thread issued before it has run;
- TMA loads and cp.async copies land in any order.
A random scheduler interleaves the roles and the asynchronous completions.  The test checks:

* every parity wait is evaluated only while its barrier has completed exactly the intended
  number of phases or one more, so the parity cannot alias;
* no TMEM buffer, ring stage, outer-tile buffer, LSE/D stage or accumulator is written
  while an earlier tile or unit may still read it, and nothing is read before it is written;
* no interleaving deadlocks, and every role finishes.

The number of warps per P/dS group is a parameter: two per group exercise the same
orderings as the kernel's eight (the barriers count warps).
"""
import random

import pytest


class Bar:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phases = 0  # completed phases

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.phases += 1
            self.pending = self.count

    def arrive(self, n=1):
        assert self.pending >= n, "more arrivals than the phase expects"
        self.pending -= n
        self._check()

    def arrive_expect_tx(self, nbytes):
        self.tx += nbytes
        self.arrive()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        assert self.tx >= 0
        self._check()


class Wait:
    """Wait for phase `k` (0-based) of `bar` by parity k & 1, as mbar_wait does."""

    def __init__(self, bar, k, what):
        self.bar, self.k, self.what = bar, k, what

    def ready(self):
        ph = self.bar.phases
        assert self.k <= ph <= self.k + 1, f"{self.what}: waiting for phase {self.k} with {ph} completed (aliased)"
        return (ph & 1) != (self.k & 1)


class Cta:
    def __init__(self, units, nb, stages, nx, km, warps_per_group, rng, skip=()):
        self.units, self.nb, self.S, self.nx, self.km = units, nb, stages, nx, km
        self.skip = set(skip)  # waits left out (to check that the model notices)
        self.W = warps_per_group
        self.rng = rng
        self.bar_x = [Bar(1) for _ in range(nx)]
        self.x_free = [Bar(1) for _ in range(nx)]
        self.s_full = [Bar(1) for _ in range(nb)]
        self.p_full = [Bar(warps_per_group) for _ in range(nb)]
        self.buf_free = [Bar(1) for _ in range(nb)]
        self.acc_full = Bar(1)
        self.acc_free = Bar(2 * warps_per_group)
        self.bar_y = [Bar(1) for _ in range(stages)]
        self.st_full = [Bar(1) for _ in range(stages)]
        self.stage_free = [Bar(1) for _ in range(stages)]
        # asynchronous work: per-issuer in-order queues, and copies that land in any order
        self.q_s, self.q_a = [], []
        self.copies = []
        # what has happened
        self.y_landed, self.x_landed, self.st_landed = set(), set(), set()
        self.s_done, self.acc_done = set(), set()
        self.pds_read = {}        # tile -> warps that read S/dP (and the stats)
        self.pds_written = {}     # tile -> warps that wrote P/dS
        self.epi_done = {}        # unit -> warps that read the accumulators
        self.unit_of_tile = []
        self.first_tile = []
        for k, T in enumerate(units):
            self.first_tile.append(len(self.unit_of_tile))
            self.unit_of_tile += [k] * T
        self.acc_mmas_left = list(units)  # accumulating MMAs of each unit not yet run

    def wait(self, bar, k, what):
        if what not in self.skip:
            yield Wait(bar, k, what)

    # ---------------------------------------------------------------- roles
    def s_issuer(self):
        g = 0
        for k, T in enumerate(self.units):
            xb = k % self.nx
            yield from self.wait(self.bar_x[xb], k // self.nx, "S: bar_x")
            for _ in range(T):
                if g >= self.nb:
                    yield from self.wait(self.buf_free[g % self.nb], (g - self.nb) // self.nb, "S: buf_free")
                yield from self.wait(self.bar_y[g % self.S], g // self.S, "S: bar_y")
                self.q_s.append(("S", g, k))
                self.q_s.append(("commit", self.s_full[g % self.nb]))
                g += 1
            self.q_s.append(("commit", self.x_free[xb]))

    def acc_issuer(self):
        g = 0
        for k, T in enumerate(self.units):
            if k >= 1:
                yield from self.wait(self.acc_free, k - 1, "acc: acc_free")
            for _ in range(T):
                yield from self.wait(self.p_full[g % self.nb], g // self.nb, "acc: p_full")
                yield from self.wait(self.bar_y[g % self.S], g // self.S, "acc: bar_y")
                self.q_a.append(("acc", g, k))
                self.q_a.append(("commit", self.buf_free[g % self.nb]))
                self.q_a.append(("commit", self.stage_free[g % self.S]))
                g += 1
            self.q_a.append(("commit", self.acc_full))

    def producer(self):
        g = 0
        for k, T in enumerate(self.units):
            xb = k % self.nx
            if k >= self.nx:
                yield from self.wait(self.x_free[xb], (k - self.nx) // self.nx, "producer: x_free")
                # every S MMA of the unit that used this buffer has run
                assert all(t in self.s_done for t in range(self.first_tile[k - self.nx],
                                                            self.first_tile[k - self.nx] + self.units[k - self.nx])), \
                    "outer-tile buffer reloaded while read"
            self.bar_x[xb].arrive_expect_tx(2)
            self.copies.append(("x", k, xb))
            for _ in range(T):
                if g >= self.S:
                    yield from self.wait(self.stage_free[g % self.S], (g - self.S) // self.S, "producer: stage_free")
                    old = g - self.S
                    assert old in self.s_done and old in self.acc_done, "ring stage refilled while read"
                    assert len(self.pds_read.get(old, ())) == self.W, "LSE/D stage refilled while read"
                self.bar_y[g % self.S].arrive_expect_tx(2)
                self.copies.append(("y", g))
                if self.km:
                    self.copies.append(("st", g))
                g += 1

    def pds_warp(self, grp, warp):
        g = 0
        for k, T in enumerate(self.units):
            for _ in range(T):
                if g % 2 == grp:
                    yield from self.wait(self.s_full[g % self.nb], g // self.nb, "P/dS: s_full")
                    if self.km:
                        yield from self.wait(self.st_full[g % self.S], g // self.S, "P/dS: st_full")
                        assert g in self.st_landed, "LSE/D read before it landed"
                    assert g in self.s_done, "S/dP read before the MMAs ran"
                    self.pds_read.setdefault(g, set()).add(warp)
                    self.pds_written.setdefault(g, set()).add(warp)
                    self.p_full[g % self.nb].arrive()
                g += 1
            yield from self.wait(self.acc_full, k, "P/dS: acc_full")
            assert self.acc_mmas_left[k] == 0, "accumulators read before the unit's MMAs ran"
            self.epi_done.setdefault(k, set()).add((grp, warp))
            self.acc_free.arrive()

    # ---------------------------------------------------------------- asynchronous work
    def run_mma(self, q):
        op = q.pop(0)
        if op[0] == "commit":
            op[1].arrive()
            return
        kind, g, k = op
        if kind == "S":
            assert g in self.y_landed and k in self.x_landed, "S MMA before its tiles landed"
            if g >= self.nb:
                old = g - self.nb
                assert old in self.acc_done, "S/dP buffer overwritten before its accumulating MMAs ran"
            self.s_done.add(g)
        else:
            assert len(self.pds_written.get(g, ())) == self.W, "accumulating MMA before P/dS was written"
            assert g in self.y_landed
            if g == self.first_tile[k] and k >= 1:
                assert len(self.epi_done.get(k - 1, ())) == 2 * self.W, "accumulators overwritten before read out"
            self.acc_mmas_left[k] -= 1
            self.acc_done.add(g)

    def land(self, i):
        c = self.copies.pop(i)
        if c[0] == "x":
            self.x_landed.add(c[1])
            self.bar_x[c[2]].complete_tx(2)
        elif c[0] == "y":
            self.y_landed.add(c[1])
            self.bar_y[c[1] % self.S].complete_tx(2)
        else:
            self.st_landed.add(c[1])
            self.st_full[c[1] % self.S].arrive()

    def simulate(self):
        agents = [self.s_issuer(), self.acc_issuer(), self.producer()]
        agents += [self.pds_warp(grp, grp * self.W + w) for grp in (0, 1) for w in range(self.W)]
        waits = [None] * len(agents)
        live = list(range(len(agents)))

        def step(i):
            try:
                waits[i] = next(agents[i])
            except StopIteration:
                live.remove(i)

        # a random speed per agent, MMA queue and kind of copy, so that some interleavings
        # leave one role far behind the others
        speeds = [0.01, 0.1, 1.0, 1.0, 10.0]
        w_agent = [self.rng.choice(speeds) for _ in agents]
        w_qs, w_qa = self.rng.choice(speeds), self.rng.choice(speeds)
        w_copy = {kind: self.rng.choice(speeds) for kind in ("x", "y", "st")}
        for i in list(live):
            step(i)
        while live or self.q_s or self.q_a or self.copies:
            choices = [("agent", i) for i in live if waits[i] is None or waits[i].ready()]
            weights = [w_agent[i] for _, i in choices]
            if self.q_s:
                choices.append(("q", self.q_s))
                weights.append(w_qs)
            if self.q_a:
                choices.append(("q", self.q_a))
                weights.append(w_qa)
            for j, c in enumerate(self.copies):
                choices.append(("copy", j))
                weights.append(w_copy[c[0]])
            assert choices, "deadlock: " + ", ".join(waits[i].what for i in live if waits[i] is not None)
            kind, x = self.rng.choices(choices, weights)[0]
            if kind == "agent":
                waits[x] = None
                step(x)
            elif kind == "q":
                self.run_mma(x)
            else:
                self.land(x)
        n = sum(self.units)
        assert self.s_done == set(range(n)) and self.acc_done == set(range(n))
        assert all(len(self.epi_done[k]) == 2 * self.W for k in range(len(self.units)))


# (NB, stages, outer buffers, key-major) of the kernel's instantiations: d = 64 (3, 8, 2),
# d = 128 dQ (3, 4, 1), d = 128 dK/dV (2, 4, 1); plus tighter rings than the kernel uses
CONFIGS = [(3, 8, 2, False), (3, 8, 2, True), (3, 4, 1, False), (2, 4, 1, True),
           (2, 2, 1, False), (3, 3, 2, True), (2, 3, 2, True)]


@pytest.mark.parametrize("nb,stages,nx,km", CONFIGS)
def test_backward_barrier_protocol(nb, stages, nx, km):
    rng = random.Random(nb * 1000 + stages * 10 + nx + (500 if km else 0))
    for _ in range(60):
        units = [rng.choice([1, 1, 2, 3, 5, 12]) for _ in range(rng.randint(1, 5))]
        Cta(units, nb, stages, nx, km, warps_per_group=2, rng=rng).simulate()


# Every wait but one is needed for ordering: the accumulate issuer's wait on the ring stage
# follows from its wait on P/dS (whose S/dP MMAs read the stage), and is there so that the
# thread issuing the MMAs has itself observed the copy's completion.
NEEDED = ["S: bar_x", "S: buf_free", "S: bar_y", "acc: acc_free", "acc: p_full", "producer: x_free",
          "producer: stage_free", "P/dS: s_full", "P/dS: st_full", "P/dS: acc_full"]


@pytest.mark.parametrize("what", NEEDED)
def test_the_model_notices_a_missing_wait(what):
    """Sanity check of the checker: with any one wait left out, some interleaving breaks an
    ordering (or aliases a phase, or deadlocks)."""
    rng = random.Random(sum(map(ord, what)))
    caught = 0
    for _ in range(60):
        units = [rng.choice([1, 2, 3, 5, 12]) for _ in range(rng.randint(2, 5))]
        try:
            Cta(units, 3, 8, 2, True, warps_per_group=2, rng=rng, skip={what}).simulate()
        except AssertionError:
            caught += 1
    assert caught > 0
