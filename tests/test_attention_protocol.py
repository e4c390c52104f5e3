"""The hand-off protocol of the tcgen05 attention template (``lower/attention.py``), model-checked
on the CPU.

One CTA's roles run as actors under a seeded random scheduler: the softmax warps, the MMA warp,
the tensor core (it executes the issued products and commits in issue order, whenever it is
scheduled), and the loaders -- either the register path (warps 5-7 store hi and lo tiles) or
the TMA path (the producer's copies complete in any order on a copy engine, the workers write
the lo tiles). Every mbarrier keeps an arrival count, a transaction count and a phase counter;
a wait names the phase it means (the template's block counter J: pair barrier J & 1, phase
J >> 1) and is satisfied only once that phase has completed. The model checks that

* no wait ever sees its barrier two phases away from the phase it means (parity aliasing),
* every S, kt, v, P, O and Q access finds the block's data, and nothing is overwritten before
  its last reader is done (S buffers, kt/v tile buffers, the one P, O across work items, the
  next item's Q while S products of the current one are pending),
* nothing deadlocks,

for 1-4 key blocks, 1-3 work items per CTA, one or two tile buffers (one: the split products
around the lo pass) and both load paths. The orders of waits and arrivals mirror the emitted
roles: ``_softmax_role``, ``_mma_role``, ``_load_lsu`` and ``_load_tma``.
"""

import random

import pytest

NLOAD, NWORK, NSOFT = 96, 64, 128


class Bar:
    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending, self.tx, self.phase = count, 0, 0

    def arrive(self, n=1, tx=0):
        self.tx += tx
        self.pending -= n
        assert self.pending >= 0, f"{self.name}: more arrivals than its count"
        self._complete()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        assert self.tx >= 0, f"{self.name}: transaction bytes below zero"
        self._complete()

    def _complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, k):
        """try_wait.parity for phase k: the hardware compares parities only."""
        assert self.phase in (k, k + 1), (
            f"{self.name}: a wait for phase {k} sees phase {self.phase} (parity aliasing)")
        return self.phase == k + 1


class Model:
    def __init__(self, NB, items, NBUF, tma, seed, bug=None):
        self.NB, self.items, self.NBUF, self.tma, self.bug = NB, items, NBUF, tma, bug
        self.split = tma and NBUF == 1
        self.rng = random.Random(seed)
        go = NLOAD + NSOFT
        self.bars = {}
        for n, cnt in (("SGO", go), ("SFULL", 1), ("PVGO", go), ("PVDONE", 1), ("KRAW", 1),
                       ("VRAW", 1), ("KLO", NWORK), ("VLO", NWORK)):
            for b in (0, 1):
                self.bars[f"{n}{b}"] = Bar(f"{n}{b}", cnt)
        self.bars["QREADY"] = Bar("QREADY", NSOFT)
        self.tq = []                    # tensor core queue: products and commits, issue order
        self.copies = []                # TMA copies in flight: (tile, block)
        # data state
        self.S = [None, None]           # block whose S is in buffer b
        self.s_read = set()             # blocks whose S the softmax has read
        self.s_done = {}                # block -> number of its S products executed
        self.pv_done = {}
        self.kraw = [None] * NBUF
        self.klo = [None] * NBUF
        self.vraw = [None] * NBUF
        self.vlo = [None] * NBUF
        self.P = None
        self.O = None                   # (item, last block accumulated)
        self.o_read = set()             # items whose O the epilogue has read
        self.Q = None                   # item whose Q is in tensor memory
        self.parts = 2 if self.split else 1     # products per S / P*V issue

    # ------------------------------------------------------------------ helpers
    def item_of(self, X):
        return X // self.NB

    def wait(self, name, X):
        """Generator: wait for phase X >> 1 of pair barrier name + (X & 1)."""
        bar = self.bars[f"{name}{X & 1}"]
        while not bar.done(X >> 1):
            yield "blocked"

    def wait_phase(self, name, k):
        bar = self.bars[name]
        while not bar.done(k):
            yield "blocked"

    def arrive(self, name, X, n, tx=0):
        self.bars[f"{name}{X & 1}"].arrive(n, tx)

    # ------------------------------------------------------------------ tensor core
    def tensor(self):
        while True:
            if not self.tq:
                yield "idle"
                continue
            op = self.tq.pop(0)
            kind = op[0]
            if kind == "commit":
                self.bars[op[1]].arrive(1)
            elif kind == "S":
                _, X, part = op
                b, kb = X & 1, X % self.NBUF
                assert self.Q == self.item_of(X), f"S_{X} without its item's Q"
                if part in (0, None):
                    assert self.kraw[kb] == X, f"S_{X} reads kt raw tile of {self.kraw[kb]}"
                if part in (1, None):
                    assert self.klo[kb] == X, f"S_{X} reads kt lo tile of {self.klo[kb]}"
                if part in (0, None):     # the first product of S_X writes the buffer
                    prev = self.S[b]
                    assert prev is None or prev in self.s_read, (
                        f"S_{X} overwrites S_{prev} before the softmax read it")
                    self.S[b] = X
                self.s_done[X] = self.s_done.get(X, 0) + 1
            elif kind == "PV":
                _, X, part = op
                vb = X % self.NBUF
                assert self.P == X, f"PV_{X} reads P of {self.P}"
                if part in (0, None):
                    assert self.vraw[vb] == X, f"PV_{X} reads v raw tile of {self.vraw[vb]}"
                if part in (1, None):
                    assert self.vlo[vb] == X, f"PV_{X} reads v lo tile of {self.vlo[vb]}"
                item = self.item_of(X)
                if X % self.NB == 0 and part in (0, None):
                    prev = self.O[0] if self.O else None
                    assert prev is None or prev in self.o_read, (
                        f"PV_{X} starts item {item}'s O before item {prev}'s was read")
                    self.O = (item, X)
                else:
                    assert self.O == (item, X - 1) or self.O == (item, X), f"O out of order at PV_{X}"
                    self.O = (item, X)
                self.pv_done[X] = self.pv_done.get(X, 0) + 1
            yield "ran"

    # ------------------------------------------------------------------ MMA warp
    def mma(self):
        J = 0
        for icount in range(self.items):
            yield from self.wait_phase("QREADY", icount)
            for j in range(self.NB):
                yield from self.issue_s(J)
                if j > 0:
                    yield from self.issue_pv(J - 1)
                J += 1
            yield from self.issue_pv(J - 1)

    def issue_s(self, J):
        yield from self.wait("SGO", J)
        if self.split:
            yield from self.wait("KRAW", J)
            self.tq.append(("S", J, 0))
            yield "step"
            yield from self.wait("KLO", J)
            self.tq.append(("S", J, 1))
        else:
            self.tq.append(("S", J, None))
        self.tq.append(("commit", f"SFULL{J & 1}"))
        yield "step"

    def issue_pv(self, J):
        yield from self.wait("PVGO", J)
        if self.split:
            yield from self.wait("VRAW", J)
            self.tq.append(("PV", J, 0))
            yield "step"
            yield from self.wait("VLO", J)
            self.tq.append(("PV", J, 1))
        else:
            self.tq.append(("PV", J, None))
        self.tq.append(("commit", f"PVDONE{J & 1}"))
        yield "step"

    # ------------------------------------------------------------------ softmax warps
    def softmax(self):
        for b in (0, 1):                        # neither S buffer holds an unread S yet
            self.arrive("SGO", b, NSOFT)
        yield "step"
        self.store_q(0, first=True)
        yield "step"
        J = 0
        for item in range(self.items):
            for j in range(self.NB):
                last = j == self.NB - 1
                if last and item + 1 < self.items and self.bug == "q_early":
                    self.store_q(item + 1)
                    yield "step"
                yield from self.wait("SFULL", J)
                if last and item + 1 < self.items and self.bug != "q_early":
                    self.store_q(item + 1)
                    yield "step"
                assert self.S[J & 1] == J and self.s_done.get(J) == self.parts, (
                    f"softmax reads S_{J} from a buffer holding S_{self.S[J & 1]}")
                self.s_read.add(J)
                self.arrive("SGO", J, NSOFT)
                yield "step"
                if j > 0 and self.rng.random() < 0.5:       # the running maximum grew
                    yield from self.wait("PVDONE", J - 1)
                    assert self.O == (item, J - 1) and self.pv_done.get(J - 1) == self.parts, (
                        f"O rescaled at block {J} while P*V_{J - 1} is pending")
                    yield "step"
                if J > 0 and self.bug != "p_without_pvdone":
                    yield from self.wait("PVDONE", J - 1)
                if self.P is not None:
                    assert self.pv_done.get(self.P) == self.parts, (
                        f"P_{J} overwrites P_{self.P} before P*V_{self.P} read it")
                self.P = J
                self.arrive("PVGO", J, NSOFT)
                yield "step"
                J += 1
            yield from self.wait("PVDONE", J - 1)
            assert self.O == (item, J - 1) and self.pv_done.get(J - 1) == self.parts, (
                f"epilogue of item {item} reads O before its last P*V")
            self.o_read.add(item)
            yield "step"

    def store_q(self, item, first=False):
        if item >= self.items:
            return
        if not first:
            last = (item * self.NB) - 1                 # the current item's last block
            assert self.s_done.get(last) == self.parts, (
                f"Q of item {item} stored while S_{last} is pending")
        self.Q = item
        self.bars["QREADY"].arrive(NSOFT)

    # ------------------------------------------------------------------ loaders
    def free_k(self, X):
        kb = X % self.NBUF
        prev = self.kraw[kb]
        if prev is not None:
            assert self.s_done.get(prev) == self.parts, (
                f"kt tile of block {X} overwrites block {prev}'s before S_{prev} read it")

    def free_v(self, X):
        vb = X % self.NBUF
        prev = self.vraw[vb]
        if prev is not None:
            assert self.pv_done.get(prev) == self.parts, (
                f"v tile of block {X} overwrites block {prev}'s before P*V_{prev} read it")

    def lsu(self):
        """Register path (``_load_lsu``): kt of block J + 1 before v of block J."""
        total = self.NB * self.items
        J = 0

        def put_k(X):
            if X >= self.NBUF and self.bug != "no_free_wait":
                yield from self.wait("SFULL", X - self.NBUF)
            self.free_k(X)
            self.kraw[X % self.NBUF] = self.klo[X % self.NBUF] = X
            self.arrive("SGO", X, NLOAD)
            yield "step"

        for item in range(self.items):
            yield from put_k(J)
            for j in range(self.NB):
                if j < self.NB - 1:
                    yield from put_k(J + 1)
                if J >= self.NBUF:
                    yield from self.wait("PVDONE", J - self.NBUF)
                self.free_v(J)
                self.vraw[J % self.NBUF] = self.vlo[J % self.NBUF] = J
                self.arrive("PVGO", J, NLOAD)
                yield "step"
                J += 1
        assert J == total

    def producer(self):
        """TMA path, warp 5 (``_load_tma``): copies complete later on the copy engine."""
        share = NLOAD if self.split else NLOAD - NWORK
        J = 0

        def issue(X, tile):
            free, raw, go = (("SFULL", "KRAW", "SGO") if tile == "k" else
                             ("PVDONE", "VRAW", "PVGO"))
            if X >= self.NBUF:
                yield from self.wait(free, X - self.NBUF)
            self.arrive(raw, X, 1, tx=1)            # expect_tx, then the copy
            self.copies.append((tile, X))
            self.arrive(go, X, share)
            yield "step"

        for item in range(self.items):
            yield from issue(J, "k")
            for j in range(self.NB):
                if j < self.NB - 1:
                    yield from issue(J + 1, "k")
                yield from issue(J, "v")
                J += 1

    def copy_engine(self):
        while True:
            if not self.copies:
                yield "idle"
                continue
            tile, X = self.copies.pop(self.rng.randrange(len(self.copies)))
            if tile == "k":
                self.free_k(X)
                self.kraw[X % self.NBUF] = X
                self.bars[f"KRAW{X & 1}"].complete_tx(1)
            else:
                self.free_v(X)
                self.vraw[X % self.NBUF] = X
                self.bars[f"VRAW{X & 1}"].complete_tx(1)
            yield "ran"

    def workers(self):
        """TMA path, warps 6-7: the lo tile once the raw tile has landed."""
        J = 0

        def lo(X, tile):
            free, raw = ("SFULL", "KRAW") if tile == "k" else ("PVDONE", "VRAW")
            go = ("KLO" if tile == "k" else "VLO") if self.split else (
                "SGO" if tile == "k" else "PVGO")
            if X >= self.NBUF:
                yield from self.wait(free, X - self.NBUF)
            yield from self.wait(raw, X)
            if tile == "k":
                assert self.kraw[X % self.NBUF] == X
                self.klo[X % self.NBUF] = X
            else:
                assert self.vraw[X % self.NBUF] == X
                self.vlo[X % self.NBUF] = X
            self.arrive(go, X, NWORK)
            yield "step"

        for item in range(self.items):
            yield from lo(J, "k")
            for j in range(self.NB):
                if j < self.NB - 1:
                    yield from lo(J + 1, "k")
                yield from lo(J, "v")
                J += 1

    # ------------------------------------------------------------------ scheduler
    def run(self):
        actors = {"softmax": self.softmax(), "mma": self.mma()}
        if self.tma:
            actors.update(producer=self.producer(), workers=self.workers())
        else:
            actors["lsu"] = self.lsu()
        daemons = {"tensor": self.tensor(), "copies": self.copy_engine()}
        steps = 0
        while actors:
            progress = False
            order = list(actors) + list(daemons)
            self.rng.shuffle(order)
            for name in order:
                gen = actors.get(name) or daemons[name]
                for _ in range(self.rng.choice([1, 1, 2, 5, 40])):
                    try:
                        r = next(gen)
                    except StopIteration:
                        actors.pop(name, None)
                        progress = True
                        break
                    if r in ("blocked", "idle"):
                        break
                    progress = True
            steps += 1
            assert progress or self.tq or self.copies, f"deadlock: {sorted(actors)} blocked"
            assert steps < 200_000, "no progress"
        # everything issued has run
        while self.tq:
            next(daemons["tensor"])
        total = self.NB * self.items
        assert all(self.s_done.get(X) == self.parts for X in range(total))
        assert all(self.pv_done.get(X) == self.parts for X in range(total))
        assert self.o_read == set(range(self.items))


@pytest.mark.parametrize("tma", [False, True], ids=["registers", "tma"])
@pytest.mark.parametrize("NBUF", [2, 1])
@pytest.mark.parametrize("NB", [1, 2, 3, 4])
def test_attention_hand_offs_hold_under_every_interleaving(NB, NBUF, tma):
    for items in (1, 2, 3):
        for seed in range(25):
            Model(NB, items, NBUF, tma, seed).run()


@pytest.mark.parametrize("bug", ["q_early", "p_without_pvdone", "no_free_wait"])
def test_the_model_finds_planted_hazards(bug):
    """Each planted change to a role's order is caught for some interleaving: storing the next
    item's Q before the last S product of the current item has landed, writing P without
    waiting for the previous P*V, and storing a kt tile without waiting for the S that reads
    the buffer's previous tile."""
    found = False
    for seed in range(300):
        try:
            Model(3, 2, 2, False, seed, bug=bug).run()
        except AssertionError:
            found = True
            break
    assert found, bug
