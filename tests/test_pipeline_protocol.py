"""A model of the persistent kernel's synchronisation protocol, run on the CPU.

attn_fwd.cuh runs five roles per CTA (producer warp 8, waiter warp 10, MMA warp 9, and
two softmax warpgroups of four warps) over a sequence of work items, with every phase
derived from running counters.  A mistake in that bookkeeping hangs or corrupts the GPU
kernel, so this file restates each role's schedule as a Python generator and runs them
under random interleavings, with:

* named barriers (ids and thread counts as in the kernel: 3 = waiter -> MMA release,
  64 threads; 4 + 2*tile + half = P half published and 8 + tile = O read out, 160
  threads; `bar.arrive` does not block, `bar.sync` waits for the generation);
* mbarriers as completion counters, where a parity wait for completion k must find the
  count at k or k + 1 (anything else would alias another phase);
* TMA copies landing and tcgen05 work completing asynchronously, the MMAs and commits of
  the MMA thread in issue order.

It checks that every schedule ends (no deadlock), that no named barrier is left with
arrivals, and the buffer hazards: S read before it is overwritten, P consumed before the
next S, O read out before the next item's first PV, K/V slots and Q reloaded only after
their readers completed.  Planted mistakes in the model (a missing O wait, a missing
Q_EMPTY wait, a missing commit) must be caught.  The model follows the kernel's
wave_item order and its ring arithmetic: the producer and waiter count ring positions,
the MMA warp uses the item's ring phase b.
"""

from __future__ import annotations

import random

import pytest

STAGES = 4


class Model:
    def __init__(self, seq, rnd, fault=None):
        self.seq = seq              # n_tiles of each item of this CTA, in order
        self.rnd = rnd
        self.fault = fault
        self.count = {}             # mbarrier -> completions
        self.nb = {3: [64, 0, 0], 4: [160, 0, 0], 5: [160, 0, 0], 6: [160, 0, 0], 7: [160, 0, 0],
                   8: [160, 0, 0], 9: [160, 0, 0]}   # id -> [threads, arrived, generation]
        self.copies = []            # landing TMA copies (callables)
        self.pipe = []              # MMA thread's async work in issue order
        self.q_item = None
        self.slot = [None] * STAGES
        self.s_buf = [None, None]
        self.o_buf = [None, None]
        self.p_done = {}
        self.o_read = {}
        self.errors = []

    # ---- primitives
    def completions(self, name):
        return self.count.get(name, 0)

    def complete(self, name):
        self.count[name] = self.completions(name) + 1

    def wait(self, name, k):
        def ready():
            c = self.completions(name)
            if c not in (k, k + 1):
                self.errors.append(f"parity alias on {name}: waiting for #{k}, {c} completions")
            return c >= k + 1
        return ready

    def arrive(self, bar_id, warps=1):
        b = self.nb[bar_id]
        b[1] += 32 * warps
        if b[1] > b[0]:
            self.errors.append(f"named barrier {bar_id} over-arrived")
        if b[1] == b[0]:
            b[1] = 0
            b[2] += 1

    def sync(self, bar_id):
        b = self.nb[bar_id]
        gen = b[2]
        self.arrive(bar_id)
        return lambda: b[2] > gen

    # ---- roles
    def producer(self):
        tt = nq = 0
        for it, n in enumerate(self.seq):
            if n == 0:
                continue
            if nq > 0:
                if self.fault != "no_q_empty_wait":
                    yield self.wait("Q_EMPTY", nq - 1)
                yield self.wait("Q", nq - 1)

            def land_q(it=it):
                self.q_item = it
                self.complete("Q")
            self.copies.append(land_q)
            nq += 1
            for lt in range(2 * n):
                slot, use = tt % STAGES, tt // STAGES
                if use > 0:
                    yield self.wait(f"KV_EMPTY{slot}", use - 1)
                    yield self.wait(f"KV_FULL{slot}", use - 1)

                def land(slot=slot, tag=(it, lt)):
                    self.slot[slot] = tag
                    self.complete(f"KV_FULL{slot}")
                self.copies.append(land)
                tt += 1

    def waiter(self):
        tt = nq = 0
        for n in self.seq:
            if n == 0:
                continue
            yield self.wait("Q", nq)
            yield self.wait(f"KV_FULL{tt % STAGES}", tt // STAGES)
            nq += 1
            tt += 1
            yield self.sync(3)
            for j in range(n):
                yield self.wait(f"KV_FULL{tt % STAGES}", tt // STAGES)
                tt += 1
                yield self.sync(3)
                if j + 1 < n:
                    yield self.wait(f"KV_FULL{tt % STAGES}", tt // STAGES)
                    tt += 1
                    yield self.sync(3)

    def mma(self):
        b = 0
        any_item = False
        for it, n in enumerate(self.seq):
            if n == 0:
                continue
            yield self.sync(3)  # Q and K_0 resident
            self.issue_s(0, it, 0, 2 * b, 0)
            self.pipe.append(("commit", "S_FULL0"))
            self.issue_s(1, it, 0, 2 * b, 0)
            self.pipe.append(("commit", "S_FULL1"))
            self.pipe.append(("commit", f"KV_EMPTY{2 * b}"))
            if n == 1:
                self.pipe.append(("commit", "Q_EMPTY"))
            for j in range(n):
                jj = b + j
                first, more = j == 0, j + 1 < n
                sv, sk = (2 * jj + 1) % STAGES, (2 * jj + 2) % STAGES
                if j == n - 1 and n > 1 and self.fault != "no_q_empty_commit":
                    self.pipe.append(("commit", "Q_EMPTY"))   # after the loop, before the last tile
                yield self.sync(3)  # V_j resident
                if first and any_item and self.fault != "no_o_free":
                    yield self.sync(8)
                yield self.sync(4)
                self.issue_pv(0, 0, it, j, sv)
                if more:
                    yield self.sync(3)  # K_{j+1} resident
                yield self.sync(5)
                self.issue_pv(0, 1, it, j, sv)
                if not more:
                    self.pipe.append(("commit", "O_DONE0"))
                if more:
                    self.issue_s(0, it, j + 1, sk, 2 * j + 2)
                    self.pipe.append(("commit", "S_FULL0"))
                if first and any_item and self.fault != "no_o_free":
                    yield self.sync(9)
                yield self.sync(6)
                self.issue_pv(1, 0, it, j, sv)
                yield self.sync(7)
                self.issue_pv(1, 1, it, j, sv)
                if not more:
                    self.pipe.append(("commit", "O_DONE1"))
                self.pipe.append(("commit", f"KV_EMPTY{sv}"))
                if more:
                    self.issue_s(1, it, j + 1, sk, 2 * j + 2)
                    self.pipe.append(("commit", "S_FULL1"))
                    self.pipe.append(("commit", f"KV_EMPTY{sk}"))
            b ^= n & 1
            any_item = True
        if any_item:
            yield self.sync(8)
            yield self.sync(9)

    def issue_s(self, tile, it, j, slot, lt):
        def run():
            if self.q_item != it:
                self.errors.append(f"S{tile}({it},{j}) read the Q of item {self.q_item}")
            if self.slot[slot] != (it, lt):
                self.errors.append(f"S{tile}({it},{j}) read slot {slot} holding {self.slot[slot]}")
            prev = self.s_buf[tile]
            if prev is not None and not self.p_done.get((tile,) + prev, False):
                self.errors.append(f"S{tile}({it},{j}) overwrote P of {prev} before PV read it")
            self.s_buf[tile] = (it, j)
        self.pipe.append(("op", run))

    def issue_pv(self, tile, half, it, j, slot):
        def run():
            if self.slot[slot] != (it, 2 * j + 1):
                self.errors.append(f"PV{tile}({it},{j}) read slot {slot} holding {self.slot[slot]}")
            if self.s_buf[tile] != (it, j):
                self.errors.append(f"PV{tile}({it},{j}) read P of {self.s_buf[tile]}")
            prev = self.o_buf[tile]  # (item, tile, halves done) of the last PV into O
            if half == 1:
                if prev != (it, j, 0):
                    self.errors.append(f"PV{tile}({it},{j}) second half after {prev}")
            elif j == 0:
                if prev is not None and not self.o_read.get((tile, prev[0]), False):
                    self.errors.append(f"PV{tile}({it},0) overwrote O of item {prev[0]} before it was read")
            elif prev != (it, j - 1, 1):
                self.errors.append(f"PV{tile}({it},{j}) accumulated onto {prev}")
            self.o_buf[tile] = (it, j, half)
            if half:
                self.p_done[(tile, it, j)] = True
        self.pipe.append(("op", run))

    def softmax(self, tile):
        tiles_before = 0
        items_before = 0
        for it, n in enumerate(self.seq):
            for j in range(n):
                yield self.wait(f"S_FULL{tile}", tiles_before + j)
                if self.s_buf[tile] != (it, j):
                    self.errors.append(f"softmax {tile} read S of {self.s_buf[tile]}, wanted {(it, j)}")
                if j > 0 and self.o_buf[tile] != (it, j - 1, 1):   # the rare rescale reads O
                    self.errors.append(f"rescale of O{tile} at ({it},{j}) saw {self.o_buf[tile]}")
                yield lambda: True
                self.arrive(4 + 2 * tile, warps=4)
                yield lambda: True
                self.arrive(5 + 2 * tile, warps=4)
            if n > 0:
                if self.fault != "no_o_wait":
                    yield self.wait(f"O_DONE{tile}", items_before)
                if self.o_buf[tile] != (it, n - 1, 1):
                    self.errors.append(f"epilogue of O{tile} item {it} read {self.o_buf[tile]}")
                self.o_read[(tile, it)] = True
                yield lambda: True
                self.arrive(8 + tile, warps=4)
                items_before += 1
            tiles_before += n

    # ---- scheduler
    def run(self):
        roles = [self.producer(), self.waiter(), self.mma(), self.softmax(0), self.softmax(1)]
        ready = [None] * len(roles)
        done = [False] * len(roles)
        for _ in range(1_000_000):
            runnable = [r for r in range(len(roles)) if not done[r] and (ready[r] is None or ready[r]())]
            n_async = len(self.copies) + (1 if self.pipe else 0)
            if not runnable and not n_async:
                break
            pick = self.rnd.randrange(len(runnable) + n_async)
            if pick < len(runnable):
                r = runnable[pick]
                try:
                    ready[r] = next(roles[r])
                except StopIteration:
                    done[r], ready[r] = True, None
            elif pick < len(runnable) + len(self.copies):
                self.copies.pop(self.rnd.randrange(len(self.copies)))()
            else:
                kind, x = self.pipe.pop(0)
                x() if kind == "op" else self.complete(x)
            if self.errors:
                return
        if not all(done):
            self.errors.append(f"deadlock: roles {[r for r in range(len(roles)) if not done[r]]} never finish")
        left = {i: b[1] for i, b in self.nb.items() if b[1]}
        if left:
            self.errors.append(f"named barriers left with arrivals: {left}")


def cta_sequences(items, grid):
    """Each CTA's items in the kernel's order (wave_item: alternating directions)."""
    seqs = []
    for cta in range(grid):
        seq, r = [], 0
        while r * grid < len(items):
            w = r * grid + ((grid - 1 - cta) if r & 1 else cta)
            if w < len(items):
                seq.append(items[w])
            r += 1
        seqs.append(seq)
    return seqs


def run_model(items, grid, seed, fault=None):
    errors = []
    for seq in cta_sequences(items, grid):
        model = Model(seq, random.Random(seed), fault)
        model.run()
        errors += model.errors
    return errors


@pytest.mark.parametrize("items,grid", [
    ([3, 1, 2], 1),
    ([1, 1, 1, 1], 1),
    ([5, 0, 2, 1, 4], 1),     # an item without keys between items with keys
    ([2] * 7, 3),
    ([32, 30, 28, 2, 1], 2),  # causal-like decreasing lengths
    ([1], 1),
    ([0, 0, 1], 1),
    ([3, 3, 3], 1),           # odd tile counts: the ring phase flips every item
])
def test_protocol_holds_under_random_interleavings(items, grid):
    for seed in range(25):
        assert run_model(items, grid, seed) == []


def test_protocol_random_item_sequences():
    rnd = random.Random(1)
    for trial in range(150):
        items = [rnd.choice([0, 1, 1, 2, 3, 5, 8]) for _ in range(rnd.randint(1, 6))]
        assert run_model(items, 1, trial) == [], items


@pytest.mark.parametrize("fault", ["no_o_wait", "no_q_empty_wait", "no_o_free", "no_q_empty_commit"])
def test_planted_mistakes_are_caught(fault):
    caught = any(run_model([4, 4, 3], 1, seed, fault) for seed in range(25))
    assert caught, fault


@pytest.mark.parametrize("n_items,grid", [(1, 1), (7, 3), (148, 148), (1024, 148), (600, 148), (1000, 7)])
def test_wave_order_visits_every_item_once(n_items, grid):
    # wave_item(r) of attn_fwd.cuh: CTA c takes r*G + c on even waves, r*G + G-1-c on odd ones.
    seen = sorted(w for seq in cta_sequences(list(range(n_items)), grid) for w in seq)
    assert seen == list(range(n_items))
    # and the CTAs' totals differ by at most one item
    counts = [len(seq) for seq in cta_sequences(list(range(n_items)), grid)]
    assert max(counts) - min(counts) <= 1
