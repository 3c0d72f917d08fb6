"""The barrier protocol of the persistent backward kernel, checked by random interleavings.

`bwd_persistent_kernel` (tiny-transformer_b200/csrc/backward_sm100.cuh, namespace persist) runs
(b, h, key tile) items back to back in one CTA: a TMA warp, a scores issuer, an accumulate
issuer, four dQ-drain warps and eight elementwise warps, synchronised by mbarriers. This test
restates each role's loop as a Python generator (same waits, arrivals, commits, buffer uses and
phase arithmetic), runs the tensor core as an in-order queue and the TMA copies as random-delay
completions, and schedules everything at random with per-run speed skew. Checked on every run:
no deadlock; every wait finds its barrier at phase e or e + 1 (a barrier two phases ahead of a
waiter would alias its parity); every buffer (TMEM S^T, dP^T, P^T, dQ, dK/dV, shared-memory dS,
the Q/dO ring, the K/V slots and their item index) is read only after its writers finished and
rewritten only after all its readers finished. The mutation tests plant known mistakes in the
restated protocol and check that the simulation reports them.
"""
import random

import pytest

STAGES, KV_SLOTS, EW, DRAIN = 3, 2, 8, 4


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.arr, self.done = name, count, 0, 0
        self.waiters = []  # target phases of blocked waiters

    def arrive(self, sim):
        self.arr += 1
        assert self.arr <= self.count, f"{self.name}: too many arrivals"
        if self.arr == self.count:
            self.arr = 0
            self.done += 1
            for e in self.waiters:
                assert self.done <= e + 1, f"{self.name}: phase {e} waiter overtaken (done={self.done})"


class Res:
    """A buffer with versions: `writers` writes complete a version, `readers` reads free it."""
    def __init__(self, name, writers, readers):
        self.name, self.nw, self.nr = name, writers, readers
        self.ver, self.w, self.r = None, 0, 0
        self.pending = None  # version being written

    def write(self, ver):
        if self.pending != ver:
            # starting a new version: the previous one must be fully read
            assert self.ver is None or self.r >= self.nr(self.ver), \
                f"{self.name}: write {ver} before readers of {self.ver} finished ({self.r})"
            assert self.pending is None or self.w >= self.nw, f"{self.name}: overlapping versions"
            self.pending, self.w = ver, 0
        self.w += 1
        if self.w == self.nw:
            self.ver, self.r, self.pending = ver, 0, None

    def begin(self, ver):
        """An asynchronous writer (TMA) starts: the previous version must be fully read."""
        assert self.ver is None or self.r >= self.nr(self.ver), \
            f"{self.name}: copy {ver} issued before readers of {self.ver} finished ({self.r})"
        assert self.pending is None
        self.pending, self.w = ver, 0

    def read(self, ver):
        assert self.ver == ver and self.pending is None, \
            f"{self.name}: read {ver} but holds {self.ver} (pending {self.pending})"
        self.r += 1


class Sim:
    # Protocol switches; the defaults are the kernel's protocol, the others plant mistakes.
    def __init__(self, items, seed, drain_releases_slot=True, wait_acc_empty=True,
                 dp_waits_ds_ready=True, q_empty_by_accumulate=True, epilogue_first=False):
        # epilogue_first: the drain warps read an item's dK/dV before draining its last dQ step
        # (an ordering the kernel could adopt; checked here ahead of any change to it).
        self.epilogue_first = epilogue_first
        self.drain_releases_slot = drain_releases_slot
        self.wait_acc_empty = wait_acc_empty
        self.dp_waits_ds_ready = dp_waits_ds_ready
        self.q_empty_by_accumulate = q_empty_by_accumulate
        self.rng = random.Random(seed)
        self.items = items
        self.counter = 0
        B = lambda n, c: Bar(n, c)
        self.bars = {n: B(n, c) for n, c in [
            ("s_full", 1), ("s_consumed", EW), ("p_full", EW), ("pv_free", 1), ("dp_full", 1),
            ("ds_ready", EW), ("ds_free", 1), ("dq_full", 1), ("dq_free", 4), ("acc_final", 1),
            ("acc_empty", 4)]}
        for i in range(KV_SLOTS):
            self.bars[f"kv_full{i}"] = Bar(f"kv_full{i}", 1)
            self.bars[f"kv_empty{i}"] = Bar(f"kv_empty{i}",
                                            1 + (DRAIN if drain_releases_slot else 0))
        for i in range(STAGES):
            self.bars[f"q_full{i}"] = Bar(f"q_full{i}", 1)
            self.bars[f"q_empty{i}"] = Bar(f"q_empty{i}", 1)
        one = lambda v: 1
        self.res = {
            "ST": Res("ST", 1, lambda v: EW), "DPT": Res("DPT", 1, lambda v: EW),
            "PT": Res("PT", EW, one), "DQ": Res("DQ", 1, lambda v: DRAIN),
            "DS": Res("DS", EW, lambda v: 2),
            "ACC": Res("ACC", 1, lambda v: DRAIN if v[0] == "fin" else 0),
        }
        for i in range(STAGES):  # Q/dO/LSE/D stage: S, dP, dV, dK MMAs + 16 EW reads
            self.res[f"Q{i}"] = Res(f"Q{i}", 1, lambda v: 4 + 2 * EW)
        self.kv_reads = {}
        for i in range(KV_SLOTS):  # K/V slot: S, dP, dQ per step of the item
            self.res[f"KV{i}"] = Res(f"KV{i}", 1, lambda v: 3 * self.kv_reads[v])
            self.res[f"IT{i}"] = Res(f"IT{i}", 1, lambda v: 2 + EW + DRAIN)
        self.item_val = [None] * KV_SLOTS
        self.fifo, self.mma_seq, self.mma_done = [], 0, 0
        self.commits = []  # (seq, bar)
        self.inflight = []  # TMA: (bar, writes)

    # -- agents -------------------------------------------------------------------------------
    def mma(self, thread, name, reads, writes):
        self.mma_seq += 1
        self.fifo.append((self.mma_seq, name, reads, writes))
        self.last_mma[thread] = self.mma_seq

    def commit(self, thread, bar):
        self.commits.append((self.last_mma.get(thread, 0), bar))
        self.flush_commits()

    def flush_commits(self):
        keep = []
        for seq, bar in self.commits:
            if seq <= self.mma_done:
                self.bars[bar].arrive(self)
            else:
                keep.append((seq, bar))
        self.commits = keep

    def tensor_step(self):
        seq, name, reads, writes = self.fifo.pop(0)
        for r in reads:
            self.res[r[0]].read(r[1])
        for w in writes:
            self.res[w[0]].write(w[1])
        self.mma_done = seq
        self.flush_commits()

    # -- roles (mirroring the kernel) ---------------------------------------------------------
    def producer(self):
        g = 0
        j = 0
        while True:
            slot = j & 1
            if j >= KV_SLOTS:
                yield ("wait", f"kv_empty{slot}", (j >> 1) - 1)
            idx = self.counter
            self.counter += 1
            if idx >= len(self.items):
                self.res[f"IT{slot}"].write(("end", j))
                self.item_val[slot] = -1
                self.bars[f"kv_full{slot}"].arrive(self)
                return
            self.res[f"IT{slot}"].write(("item", j))
            self.item_val[slot] = idx
            self.kv_reads[("kv", j)] = self.items[idx]
            self.res[f"KV{slot}"].begin(("kv", j))
            self.inflight.append((f"kv_full{slot}", [(f"KV{slot}", ("kv", j))]))
            for i in range(self.items[idx]):
                st = g % STAGES
                if g >= STAGES:
                    yield ("wait", f"q_empty{st}", (g // STAGES) - 1)
                self.res[f"Q{st}"].begin(("q", g))
                self.inflight.append((f"q_full{st}", [(f"Q{st}", ("q", g))]))
                g += 1
            j += 1

    def read_item(self, slot, j):
        self.res[f"IT{slot}"].read(("end", j) if self.item_val[slot] == -1 else ("item", j))
        return self.item_val[slot]

    def scores(self):
        g = 0
        j = 0
        while True:
            slot = j & 1
            yield ("wait", f"kv_full{slot}", j >> 1)
            idx = self.read_item(slot, j)
            if idx < 0:
                return
            for i in range(self.items[idx]):
                st = g % STAGES
                yield ("wait", f"q_full{st}", g // STAGES)
                if g > 0:
                    yield ("wait", "s_consumed", g - 1)
                self.mma("sc", "S", [(f"Q{st}", ("q", g)), (f"KV{slot}", ("kv", j))], [("ST", g)])
                self.commit("sc", "s_full")
                if g > 0 and self.dp_waits_ds_ready:
                    yield ("wait", "ds_ready", g - 1)
                self.mma("sc", "dP", [(f"Q{st}", ("q", g)), (f"KV{slot}", ("kv", j))], [("DPT", g)])
                self.commit("sc", "dp_full")
                g += 1
            j += 1

    def accum(self):
        g = 0
        j = 0
        while True:
            slot = j & 1
            yield ("wait", f"kv_full{slot}", j >> 1)
            idx = self.read_item(slot, j)
            if idx < 0:
                return
            n = self.items[idx]
            for i in range(n):
                st = g % STAGES
                yield ("wait", "p_full", g)
                if i == 0 and j > 0 and self.wait_acc_empty:
                    yield ("wait", "acc_empty", j - 1)
                self.mma("ac", "dV", [("PT", g), (f"Q{st}", ("q", g))],
                         [("ACC", ("first", j))] if i == 0 else [])
                self.commit("ac", "pv_free")
                yield ("wait", "ds_ready", g)
                self.mma("ac", "dK", [("DS", g), (f"Q{st}", ("q", g))],
                         [("ACC", ("fin", j))] if i + 1 == n else [])
                self.commit("ac" if self.q_empty_by_accumulate else "sc", f"q_empty{st}")
                if i + 1 == n:
                    self.commit("ac", "acc_final")
                if g > 0:
                    yield ("wait", "dq_free", g - 1)
                self.mma("ac", "dQ", [("DS", g), (f"KV{slot}", ("kv", j))], [("DQ", g)])
                self.commit("ac", "dq_full")
                self.commit("ac", "ds_free")
                if i + 1 == n:
                    self.commit("ac", f"kv_empty{slot}")
                g += 1
            j += 1

    def drain(self, w):
        g = 0
        j = 0
        while True:
            slot = j & 1
            yield ("wait", f"kv_full{slot}", j >> 1)
            idx = self.read_item(slot, j)
            if self.drain_releases_slot:
                self.bars[f"kv_empty{slot}"].arrive(self)
            if idx < 0:
                return
            n = self.items[idx]
            for i in range(n):
                if i + 1 == n and self.epilogue_first:
                    yield from self.epilogue(j)
                yield ("wait", "dq_full", g)
                self.res["DQ"].read(g)
                self.bars["dq_free"].arrive(self)
                g += 1
            if not self.epilogue_first:
                yield from self.epilogue(j)
            j += 1

    def epilogue(self, j):
        yield ("wait", "acc_final", j)
        self.res["ACC"].read(("fin", j))
        self.bars["acc_empty"].arrive(self)

    def ew(self, w):
        g = 0
        j = 0
        while True:
            slot = j & 1
            yield ("wait", f"kv_full{slot}", j >> 1)
            idx = self.read_item(slot, j)
            if idx < 0:
                return
            for i in range(self.items[idx]):
                st = g % STAGES
                yield ("wait", "s_full", g)
                self.res["ST"].read(g)
                self.bars["s_consumed"].arrive(self)
                if g > 0:
                    yield ("wait", "pv_free", g - 1)
                self.res[f"Q{st}"].read(("q", g))  # LSE rows
                self.res["PT"].write(g)
                self.bars["p_full"].arrive(self)
                yield ("wait", "dp_full", g)
                self.res["DPT"].read(g)
                if g > 0:
                    yield ("wait", "ds_free", g - 1)
                self.res[f"Q{st}"].read(("q", g))  # D rows
                self.res["DS"].write(g)
                self.bars["ds_ready"].arrive(self)
                g += 1
            j += 1

    # -- scheduler ----------------------------------------------------------------------------
    def run(self):
        self.last_mma = {}
        roles = [("prod", self.producer()), ("sc", self.scores()), ("ac", self.accum())]
        roles += [(f"dr{w}", self.drain(w)) for w in range(DRAIN)]
        roles += [(f"ew{w}", self.ew(w)) for w in range(EW)]
        state = {n: None for n, _ in roles}  # pending wait
        gens = dict(roles)
        alive = set(gens)
        # per-run speeds: some roles or agents run much slower than others
        speed = {n: self.rng.choice([0.02, 0.2, 1.0]) for n in list(gens) + ["tensor", "tma"]}
        steps = 0
        while alive or self.fifo or self.inflight:
            steps += 1
            assert steps < 10 ** 7
            choices = []
            for n in alive:
                wt = state[n]
                if wt is None or self.bars[wt[0]].done >= wt[1] + 1:
                    choices.append(("role", n))
            if self.fifo:
                choices.append(("tensor", None))
            for k in range(len(self.inflight)):
                choices.append(("tma", k))
            if not choices:
                raise AssertionError(f"deadlock: waits {[(n, state[n]) for n in alive]}")
            weights = [speed.get(c[1] if c[0] == "role" else c[0], 1.0) for c in choices]
            kind, arg = self.rng.choices(choices, weights)[0]
            if kind == "tensor":
                self.tensor_step()
            elif kind == "tma":
                bar, writes = self.inflight.pop(arg)
                for r, v in writes:
                    self.res[r].write(v)
                self.bars[bar].arrive(self)
            else:
                n = arg
                if state[n] is not None:
                    bar = self.bars[state[n][0]]
                    bar.waiters.remove(state[n][1])
                    state[n] = None
                try:
                    op = next(gens[n])
                except StopIteration:
                    alive.discard(n)
                    continue
                assert op[0] == "wait"
                bar, e = self.bars[op[1]], op[2]
                assert bar.done in (e, e + 1), f"{n}: waits {op[1]} phase {e}, done={bar.done}"
                if bar.done < e + 1:
                    state[n] = (op[1], e)
                    bar.waiters.append(e)
        # every item's accumulators were read, every step drained
        return steps


def random_items(seed):
    rng = random.Random(seed)
    return [rng.randint(1, 5) for _ in range(rng.randint(0, 7))]


@pytest.mark.parametrize("epilogue_first", [False, True])
def test_protocol_random_interleavings(epilogue_first):
    for seed in range(2000):
        Sim(random_items(seed), seed, epilogue_first=epilogue_first).run()


@pytest.mark.parametrize("mistake, message", [
    (dict(drain_releases_slot=False), "IT"),       # slot refilled while a drain warp lags
    (dict(wait_acc_empty=False), "ACC"),           # dV/dK overwritten before the epilogue read
    (dict(dp_waits_ds_ready=False), "DPT"),        # dP^T overwritten before phase 2 read it
    (dict(q_empty_by_accumulate=False), "Q"),      # Q stage freed before dV/dK read it
])
def test_protocol_mistakes_are_reported(mistake, message):
    for seed in range(2000):
        try:
            Sim(random_items(seed), seed, **mistake).run()
        except AssertionError as e:
            assert message in str(e)
            return
    pytest.fail(f"planted mistake {mistake} not detected")
