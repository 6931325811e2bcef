"""Model check of the forward main kernel's barrier protocol (csrc/swa_kernels.cu,
`swa_main_body`), on the CPU, in the manner of test_bwd_protocol.py.

The roles of one CTA are restated as generators following the kernel's loops and waits:
- the producer: the unit ring, the two Q buffers and the K/V slot ring;
- the two MMA issuers, one per query tile X, each with S per chain and the pending tile's
  P*V before the next S;
- the softmax warps: per query tile, H warpgroups.  H = 2 at d = 64, one per chain, each
  with its own accumulator.  H = 1 at d = 128, one warpgroup running both chains into one
  accumulator.

Each unit has random member tiles per query tile.  A query tile that is active has at least
one member tile; unit decode guarantees it, and without it the softmax would wait for an
accumulator that no P*V fills.  Rare rescales of the accumulator are drawn at random,
including the d = 128 wait on the other chain's P*V.

The model checks:
* no parity aliasing (every wait evaluated while its barrier is at the intended phase or
  the next one);
* slots and Q buffers are refilled only after every MMA reading them has run;
* S overwrites a chain's TMEM columns only after that chain's P was written and its P*V
  ran;
* P*V runs only after P is written and V landed;
* a unit's first P*V overwrites the accumulators only after the previous unit's epilogue
  read them;
* a rescale finds no P*V into its accumulator still pending;
* the epilogue reads the accumulators only after every P*V of the unit ran;
* the halves' exchange buffer is read only after both halves wrote it, and rewritten only
  after it was read;
* no interleaving deadlocks.
"""
import random

import pytest

from test_bwd_protocol import Bar, Wait


class Unit:
    def __init__(self, ntiles, active, mem):
        self.ntiles, self.active, self.mem = ntiles, active, mem


def random_units(rng, count):
    units = []
    for _ in range(count):
        nt = rng.randint(1, 6)
        active = [rng.random() < 0.9, rng.random() < 0.9]
        if not any(active):
            active[rng.randrange(2)] = True
        mem = []
        for x in range(2):
            m = [active[x] and rng.random() < 0.7 for _ in range(nt)]
            if active[x] and not any(m):
                m[rng.randrange(nt)] = True
            mem.append(m)
        units.append(Unit(nt, active, mem))
    return units


class Cta:
    def __init__(self, units, H, slots, ring, wpg, rng, rescale_p=0.2, skip=()):
        self.units, self.H, self.S, self.R, self.Wm, self.rng = units, H, slots, ring, wpg, rng
        self.NC = 2
        self.rescale_p = rescale_p
        self.skip = set(skip)
        n_sm = 2 * H * wpg  # softmax warps
        self.q_full = [Bar(1) for _ in range(2)]
        self.q_empty = [Bar(1) for _ in range(2)]
        self.s_full = [[Bar(1) for _ in range(2)] for _ in range(2)]
        self.p_full = [[Bar(wpg) for _ in range(2)] for _ in range(2)]
        self.pv_done = [[Bar(1) for _ in range(2)] for _ in range(2)]
        self.o_full = [Bar(1) for _ in range(2)]
        self.o_free = [Bar(H * wpg) for _ in range(2)]
        self.tile_bar = [Bar(H * wpg) for _ in range(2)]  # named barrier of tile X's warpgroups
        self.kv_full = [Bar(1) for _ in range(slots)]
        self.kv_empty = [Bar(2) for _ in range(slots)]
        self.unit_full = [Bar(1) for _ in range(ring)]
        self.unit_empty = [Bar(2 + n_sm) for _ in range(ring)]
        self.ring_val = [None] * ring
        self.queues = [[], []]
        self.copies = []
        # what has happened
        self.landed = set()        # ("q", x, k) / ("kv", L)
        self.s_exec = set()        # (X, h, unit, j)
        self.pv_exec = set()
        self.pv_pending = [[], []]  # per X: (h, unit, j) issued, not yet run
        self.p_written = {}        # (X, h, unit, j) -> warps
        self.epi = [{}, {}]        # per X: accumulation index -> warps that read O
        self.xchg_read = [{}, {}]  # per X: accumulation index -> warps that read the exchange
        self.xchg_written = [{}, {}]
        self.first_L = []
        L = 0
        for u in units:
            self.first_L.append(L)
            L += 2 * u.ntiles
        self.n_loads = L

    def wait(self, bar, k, what):
        if what not in self.skip:
            yield Wait(bar, k, what)

    def load_of(self, L):
        """(unit, tile, is_v) of K/V load L."""
        for u in range(len(self.units) - 1, -1, -1):
            if L >= self.first_L[u]:
                j, kv = divmod(L - self.first_L[u], 2)
                return u, j, kv

    # ---------------------------------------------------------------- roles
    def producer(self):
        L = qn = 0
        for k in range(len(self.units) + 1):
            us = k % self.R
            if k >= self.R:
                yield from self.wait(self.unit_empty[us], k // self.R - 1, "producer: unit_empty")
            self.ring_val[us] = k
            self.unit_full[us].arrive()
            if k == len(self.units):
                break
            for x in range(2):
                if qn > 0:
                    yield from self.wait(self.q_empty[x], qn - 1, "producer: q_empty")
                    pu = self.units[k - 1]
                    for j in range(pu.ntiles):
                        if pu.mem[x][j]:
                            assert all((x, h, k - 1, j) in self.s_exec for h in range(self.NC)), \
                                "Q refilled while its S MMAs may run"
                self.q_full[x].arrive_expect_tx(1)
                self.copies.append(("q", x, k))
            qn += 1
            for _ in range(self.units[k].ntiles):
                for _kv in range(2):
                    slot = L % self.S
                    if L >= self.S:
                        yield from self.wait(self.kv_empty[slot], L // self.S - 1, "producer: kv_empty")
                        u, j, isv = self.load_of(L - self.S)
                        for x in range(2):
                            if self.units[u].mem[x][j]:
                                done = self.pv_exec if isv else self.s_exec
                                assert all((x, h, u, j) in done for h in range(self.NC)), \
                                    "K/V slot refilled while an MMA may read it"
                    self.kv_full[slot].arrive_expect_tx(1)
                    self.copies.append(("kv", L))
                    L += 1
        # drain: every issued copy lands before the CTA exits
        if qn > 0:
            for x in range(2):
                yield from self.wait(self.q_full[x], qn - 1, "producer: drain q_full")
        for idx in range(max(0, L - self.S), L):
            yield from self.wait(self.kv_full[idx % self.S], idx // self.S, "producer: drain kv_full")

    def mma_issuer(self, X):
        q = self.queues[X]
        L = qn = pc = oc = 0
        for k in range(len(self.units) + 1):
            us = k % self.R
            yield from self.wait(self.unit_full[us], k // self.R, "mma: unit_full")
            u = self.ring_val[us]
            assert u == k, "unit ring read before its entry was published (or after it was reused)"
            self.unit_empty[us].arrive()
            if u >= len(self.units):
                break
            un = self.units[u]
            act = un.active[X]
            yield from self.wait(self.q_full[X], qn, "mma: q_full")
            qn += 1
            st = {"first": True, "pend": None}

            def pv_half(h):
                lv, pu, pj = st["pend"]
                if h == 0:
                    if st["first"] and oc > 0:
                        yield from self.wait(self.o_free[X], oc - 1, "mma: o_free")
                    yield from self.wait(self.kv_full[lv % self.S], lv // self.S, "mma: kv_full (V)")
                yield from self.wait(self.p_full[X][h], pc, "mma: p_full")
                fresh = st["first"] and (self.H == 2 or h == 0)
                q.append(("pv", X, h, pu, pj, fresh, oc))
                self.pv_pending[X].append((h, pu, pj))
                q.append(("commit", self.pv_done[X][h]))

            def pv_finish():
                nonlocal pc
                lv = st["pend"][0]
                pc += 1
                st["first"] = False
                q.append(("commit", self.kv_empty[lv % self.S]))
                st["pend"] = None

            for j in range(un.ntiles):
                mem = act and un.mem[X][j]
                lk = L + 2 * j
                lv = lk + 1
                if not mem:
                    if st["pend"] is not None:
                        for h in range(self.NC):
                            yield from pv_half(h)
                        pv_finish()
                    yield from self.wait(self.kv_full[lk % self.S], lk // self.S, "mma: kv_full (K)")
                else:
                    for h in range(self.NC):
                        if st["pend"] is not None:
                            yield from pv_half(h)
                        if h == 0:
                            yield from self.wait(self.kv_full[lk % self.S], lk // self.S, "mma: kv_full (K)")
                        q.append(("s", X, h, u, j))
                        q.append(("commit", self.s_full[X][h]))
                    if st["pend"] is not None:
                        pv_finish()
                if mem:
                    q.append(("commit", self.kv_empty[lk % self.S]))
                    st["pend"] = (lv, u, j)
                else:
                    self.kv_empty[lk % self.S].arrive()
                    yield from self.wait(self.kv_full[lv % self.S], lv // self.S, "mma: kv_full (V)")
                    self.kv_empty[lv % self.S].arrive()
            q.append(("commit", self.q_empty[X]))
            if st["pend"] is not None:
                for h in range(self.NC):
                    yield from pv_half(h)
                pv_finish()
            if not st["first"]:
                q.append(("commit", self.o_full[X]))
                oc += 1
            L += 2 * un.ntiles

    def softmax_warp(self, X, hh, w):
        sc = oc = 0
        chains = [hh] if self.H == 2 else [0, 1]
        for k in range(len(self.units) + 1):
            us = k % self.R
            yield from self.wait(self.unit_full[us], k // self.R, "softmax: unit_full")
            u = self.ring_val[us]
            assert u == k, "unit ring read before its entry was published (or after it was reused)"
            self.unit_empty[us].arrive()
            if u >= len(self.units):
                break
            un = self.units[u]
            if not un.active[X]:
                continue
            for j in range(un.ntiles):
                if not un.mem[X][j]:
                    continue
                for ch in chains:
                    yield from self.wait(self.s_full[X][ch], sc, "softmax: s_full")
                    assert (X, ch, u, j) in self.s_exec, "S read before its MMAs ran"
                    if self.rng.random() < self.rescale_p:
                        if self.H == 1:
                            other = 1 - ch
                            ptile = sc - 1 if ch == 0 else sc
                            yield from self.wait(self.pv_done[X][other], ptile, "softmax: pv_done (rescale)")
                            assert not self.pv_pending[X], "accumulator rescaled under a pending P*V"
                        else:
                            assert not any(h == ch for h, _, _ in self.pv_pending[X]), \
                                "accumulator rescaled under a pending P*V"
                    self.p_written.setdefault((X, ch, u, j), set()).add((hh, w))
                    self.p_full[X][ch].arrive()
                sc += 1
            yield from self.wait(self.o_full[X], oc, "softmax: o_full")
            assert not self.pv_pending[X], "accumulators read before the unit's P*V ran"
            if self.H == 2:
                # the halves exchange (m, l) through buffer oc & 1, written before the named
                # barrier and read after it
                prev = self.xchg_read[X].get(oc - 2, set())
                assert oc < 2 or len(prev) == self.H * self.Wm, "exchange buffer rewritten before read"
                self.xchg_written[X].setdefault(oc, set()).add((hh, w))
                self.tile_bar[X].arrive()
                yield from self.wait(self.tile_bar[X], oc, "softmax: tile_bar")
                assert len(self.xchg_written[X][oc]) == self.H * self.Wm, "exchange read before both halves wrote it"
                self.xchg_read[X].setdefault(oc, set()).add((hh, w))
            self.epi[X].setdefault(oc, set()).add((hh, w))
            oc += 1
            self.o_free[X].arrive()

    # ---------------------------------------------------------------- asynchronous work
    def run_op(self, X):
        op = self.queues[X].pop(0)
        if op[0] == "commit":
            op[1].arrive()
            return
        if op[0] == "s":
            _, X, h, u, j = op
            L = self.first_L[u] + 2 * j
            assert ("kv", L) in self.landed and ("q", X, u) in self.landed, "S before its tiles landed"
            # the previous member tile's P in these columns: written and consumed
            prev = [(pu, pj) for (pu, pj) in self._members(X) if (pu, pj) < (u, j)]
            if prev:
                pu, pj = prev[-1]
                assert len(self.p_written.get((X, h, pu, pj), ())) == self.Wm, "S over a P not yet written"
                assert (X, h, pu, pj) in self.pv_exec, "S over a P whose P*V has not run"
            self.s_exec.add((X, h, u, j))
        else:
            _, X, h, u, j, fresh, acc_i = op
            assert len(self.p_written.get((X, h, u, j), ())) == self.Wm, "P*V before P was written"
            assert ("kv", self.first_L[u] + 2 * j + 1) in self.landed, "P*V before V landed"
            if fresh and acc_i > 0:
                assert len(self.epi[X].get(acc_i - 1, ())) == self.H * self.Wm, \
                    "accumulators overwritten before the previous epilogue read them"
            self.pv_pending[X].remove((h, u, j))
            self.pv_exec.add((X, h, u, j))

    def _members(self, X):
        return [(u, j) for u, un in enumerate(self.units) for j in range(un.ntiles) if un.mem[X][j]]

    def land(self, i):
        c = self.copies.pop(i)
        self.landed.add(c)
        if c[0] == "q":
            self.q_full[c[1]].complete_tx(1)
        else:
            self.kv_full[c[1] % self.S].complete_tx(1)

    def simulate(self):
        agents = [self.producer(), self.mma_issuer(0), self.mma_issuer(1)]
        agents += [self.softmax_warp(X, hh, w) for X in range(2) for hh in range(self.H) for w in range(self.Wm)]
        speeds = [0.01, 0.1, 1.0, 1.0, 10.0]
        w_agent = [self.rng.choice(speeds) for _ in agents]
        w_q = [self.rng.choice(speeds) for _ in range(2)]
        w_copy = self.rng.choice(speeds)
        waits = [None] * len(agents)
        live = list(range(len(agents)))

        def step(i):
            try:
                waits[i] = next(agents[i])
            except StopIteration:
                live.remove(i)

        for i in list(live):
            step(i)
        while live or self.queues[0] or self.queues[1] or self.copies:
            choices = [("agent", i) for i in live if waits[i] is None or waits[i].ready()]
            weights = [w_agent[i] for _, i in choices]
            for X in range(2):
                if self.queues[X]:
                    choices.append(("q", X))
                    weights.append(w_q[X])
            for j in range(len(self.copies)):
                choices.append(("copy", j))
                weights.append(w_copy)
            assert choices, "deadlock: " + ", ".join(waits[i].what for i in live if waits[i] is not None)
            kind, x = self.rng.choices(choices, weights)[0]
            if kind == "agent":
                waits[x] = None
                step(x)
            elif kind == "q":
                self.run_op(x)
            else:
                self.land(x)
        for X in range(2):
            for u, j in self._members(X):
                assert all((X, h, u, j) in self.pv_exec for h in range(self.NC))


# (softmax warpgroups per tile, K/V slots) of the two instantiations, plus tighter rings
CONFIGS = [(2, 7), (1, 3), (2, 2), (1, 2), (2, 3)]


@pytest.mark.parametrize("H,slots", CONFIGS)
def test_forward_barrier_protocol(H, slots):
    rng = random.Random(H * 100 + slots)
    for _ in range(60):
        units = random_units(rng, rng.randint(1, 7))
        Cta(units, H, slots, ring=4, wpg=2, rng=rng).simulate()


def test_an_active_tile_without_member_tiles_deadlocks():
    """The invariant unit decode must keep: an active query tile has a member tile."""
    rng = random.Random(3)
    units = [Unit(2, [True, True], [[True, False], [False, False]])]
    with pytest.raises(AssertionError, match="deadlock"):
        Cta(units, 2, 7, ring=4, wpg=2, rng=rng).simulate()


NEEDED = ["producer: unit_empty", "producer: q_empty", "producer: kv_empty", "mma: unit_full", "mma: q_full",
          "mma: o_free", "mma: kv_full (V)", "mma: p_full", "mma: kv_full (K)", "softmax: unit_full",
          "softmax: s_full", "softmax: o_full", "softmax: pv_done (rescale)", "softmax: tile_bar"]


@pytest.mark.parametrize("what", NEEDED)
def test_the_model_notices_a_missing_wait(what):
    H = 1 if what == "softmax: pv_done (rescale)" else 2
    rng = random.Random(sum(map(ord, what)))
    caught = 0
    for _ in range(80):
        units = random_units(rng, rng.randint(2, 7))
        try:
            Cta(units, H, 3, ring=2 if "unit" in what else 4, wpg=2, rng=rng, rescale_p=0.5,
                skip={what}).simulate()
        except AssertionError:
            caught += 1
    assert caught > 0
