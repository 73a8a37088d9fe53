"""Host model of the warp-specialised pipeline of attn_prefill_tc_kernel
(csrc/attn_prefill_tc.cu), for protocol tests on CPU.

The model replays the kernel's synchronisation, not its arithmetic:
  - mbarriers with an arrival count, a transaction-byte count and a completed
    phase count; a wait names the logical phase it expects and passes its
    parity, as the kernel does; a wait that finds the barrier two phases on
    (the waiter was lapped, where the hardware would block on the parity) is
    an error;
  - TMA loads complete at random times, each adding its bytes to its barrier;
  - tensor-core MMAs and tcgen05.commit markers complete in issue order;
  - thread roles: the producer (warp 0), the MMA issuer (warp 1), two V
    transposer warps (2-3) and four softmax warps (4-7), each a generator
    that mirrors its branch of the kernel statement for statement;
  - every shared-memory / TMEM buffer carries the tile index last written
    into it; a reader checks it sees the tile it expects, and overlapping
    accesses of two agents where either writes are reported as races.
A seeded scheduler picks at random among the roles that can run and the async
completions that are due.  `fault_at` makes one blocked wait (one that
records an error code) give up, as a bounded wait that ran out would; any
wait left blocked with nothing else able to run then also gives up, as the
bounded waits of the kernel do.  `named_barrier=True` restores the earlier
transposer hand-off (a `bar.sync` across both transposer warps, with no time
limit, and one kv_empty arrival for both) to show the hang it allowed.
"""
from __future__ import annotations

import random
from collections import defaultdict, deque

Q_BYTES = 128 * 128 * 2
KV_BYTES = 64 * 128 * 2


class Bar:
    def __init__(self, name: str, count: int):
        self.name, self.count = name, count
        self.pending, self.tx, self.phase = count, 0, 0

    def _maybe(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, n: int = 1):
        self.pending -= n
        assert self.pending >= 0, f"{self.name}: more arrivals than its count"
        self._maybe()

    def arrive_expect_tx(self, nbytes: int):
        self.tx += nbytes
        self.arrive()

    def complete_tx(self, nbytes: int):
        self.tx -= nbytes
        self._maybe()


class Wait:
    """A parity wait for logical phase `phase`.  The hardware compares only
    the parity of the barrier's current phase, so the wait is sound only
    while the barrier has completed `phase` or `phase + 1` phases, i.e. the
    completed count c stays in {phase, phase + 1} until the wait returns: at
    c < phase the parity test would pass at once (premature), at c > phase + 1
    it would block (lapped)."""

    def __init__(self, bar: Bar, phase: int, code):
        self.bar, self.phase, self.code = bar, phase, code

    def ready(self) -> bool:
        return self.bar.phase >= self.phase + 1

    def hazard(self):
        c = self.bar.phase
        if c < self.phase:
            return (f"waits for phase {self.phase} of {self.bar.name} while it has completed "
                    f"{c} (the parity test would pass early)")
        return None


class NamedBarrier:
    """bar.sync over `threads` (no time limit)."""

    def __init__(self, parties: int):
        self.parties, self.arrived, self.gen = parties, 0, 0


class NamedWait:
    def __init__(self, nb: NamedBarrier):
        self.nb = nb
        nb.arrived += 1
        self.gen = nb.gen
        if nb.arrived == nb.parties:
            nb.arrived, nb.gen = 0, nb.gen + 1

    def ready(self) -> bool:
        return self.nb.gen > self.gen


class Model:
    def __init__(self, n_kb: int, seed: int, fault_at=None, named_barrier: bool = False):
        self.n_kb, self.rng = n_kb, random.Random(seed)
        self.fault_at, self.named = fault_at, named_barrier
        self.q_full = Bar("q_full", 1)
        self.kv_full = [Bar(f"kv_full{i}", 1) for i in range(2)]
        self.kv_empty = [Bar(f"kv_empty{i}", 2 if named_barrier else 3) for i in range(2)]
        self.s_full = [Bar(f"s_full{i}", 1) for i in range(2)]
        self.s_free = [Bar(f"s_free{i}", 128) for i in range(2)]
        self.p_full = [Bar(f"p_full{i}", 128) for i in range(2)]
        self.vt_full = [Bar(f"vt_full{i}", 64) for i in range(2)]
        self.o_full = [Bar(f"o_full{i}", 1) for i in range(2)]
        self.o_free = [Bar(f"o_free{i}", 128) for i in range(2)]
        self.mma_done = Bar("mma_done", 1)
        self.tr_bar = NamedBarrier(2)
        self.abort = False
        self.err = 0
        self.tma: list = []            # in-flight loads (agent, buf, bar, bytes, tag)
        self.pipe: deque = deque()     # ("mma", agent, reads, writes) | ("commit", bar)
        self.mem: dict = {}
        self.access = defaultdict(list)
        self.errors: list = []
        self.seen = defaultdict(list)  # softmax warp -> tiles whose O it folded in
        self._n = 0

    # ------------------------------------------------------------ accesses
    def begin(self, agent, buf, kind):
        for a, k in self.access[buf]:
            if a != agent and "w" in (k, kind):
                self.errors.append(f"race on {buf}: {agent} {kind} against {a} {k}")
        self.access[buf].append((agent, kind))

    def end(self, agent, buf, kind):
        self.access[buf].remove((agent, kind))

    def check(self, who, buf, tag):
        if self.mem.get(buf) != tag:
            self.errors.append(f"{who} read {buf} holding {self.mem.get(buf)!r}, wanted {tag!r}")

    # ------------------------------------------------------------ async units
    def tma_load(self, buf, bar, nbytes, tag):
        self._n += 1
        agent = f"tma{self._n}"
        self.begin(agent, buf, "w")
        self.tma.append((agent, buf, bar, nbytes, tag))

    def mma(self, reads, writes):
        # one agent: MMAs issued by the one MMA thread execute in issue order,
        # so two of them never overlap on a buffer (the tags still check each
        # one reads what it should)
        agent = "tensor-pipe"
        for b, _ in reads:
            self.begin(agent, b, "r")
        for b, _ in writes:
            self.begin(agent, b, "w")
        self.pipe.append(("mma", agent, reads, writes))

    def commit(self, bar):
        self.pipe.append(("commit", bar))

    def _complete_tma(self, i):
        agent, buf, bar, nbytes, tag = self.tma.pop(i)
        self.mem[buf] = tag
        self.end(agent, buf, "w")
        bar.complete_tx(nbytes)

    def _complete_pipe(self):
        op = self.pipe.popleft()
        if op[0] == "commit":
            op[1].arrive()
            return
        _, agent, reads, writes = op
        for b, tag in reads:
            self.check(agent, b, tag)
            self.end(agent, b, "r")
        for b, tag in writes:
            self.mem[b] = tag
            self.end(agent, b, "w")

    # ------------------------------------------------------------ roles
    def producer(self):
        n_kb = self.n_kb
        self.q_full.arrive_expect_tx(Q_BYTES)
        self.tma_load("Q", self.q_full, Q_BYTES, "q")
        yield None
        issued = 0
        for j in range(n_kb):
            if self.abort:
                break
            s = j & 1
            if j >= 2 and not (yield Wait(self.kv_empty[s], (j >> 1) - 1, 0x601)):
                self.abort = True
                break
            self.kv_full[s].arrive_expect_tx(2 * KV_BYTES)
            self.tma_load(f"K{s}", self.kv_full[s], KV_BYTES, j)
            self.tma_load(f"V{s}", self.kv_full[s], KV_BYTES, j)
            issued = j + 1
            yield None
        yield Wait(self.q_full, 0, None)
        for j in range(max(0, issued - 2), issued):
            yield Wait(self.kv_full[j & 1], j >> 1, None)

    def mma_issuer(self):
        n_kb = self.n_kb
        ok = yield Wait(self.q_full, 0, 0x602)

        def issue_s(j):
            s = j & 1
            if not (yield Wait(self.kv_full[s], j >> 1, 0x603)):
                return False
            if j >= 2 and not (yield Wait(self.s_free[s], (j >> 1) - 1, 0x604)):
                return False
            self.mma([("Q", "q"), (f"K{s}", j)], [(f"S{s}.{w}", j) for w in range(4)])
            self.commit(self.s_full[s])
            self.commit(self.kv_empty[s])
            return True

        if ok and n_kb > 0:
            ok = yield from issue_s(0)
        j = 0
        while ok and j < n_kb and not self.abort:
            if j + 1 < n_kb and not (yield from issue_s(j + 1)):
                ok = False
                break
            s = j & 1
            if (not (yield Wait(self.p_full[s], j >> 1, 0x605))
                    or not (yield Wait(self.vt_full[s], j >> 1, 0x606))
                    or (j >= 2 and not (yield Wait(self.o_free[s], (j >> 1) - 1, 0x607)))):
                ok = False
                break
            self.mma([(f"P{s}.{w}", j) for w in range(4)] + [(f"VT{s}.{h}", j) for h in range(2)],
                     [(f"O{s}.{w}", j) for w in range(4)])
            self.commit(self.o_full[s])
            j += 1
            yield None
        if not ok:
            self.abort = True
        self.commit(self.mma_done)
        yield Wait(self.mma_done, 0, None)

    def transposer(self, w):
        agent = f"transposer{w}"
        for j in range(self.n_kb):
            if self.abort:
                break
            s = j & 1
            if not (yield Wait(self.kv_full[s], j >> 1, 0x608)):
                self.abort = True
                break
            if j >= 2 and not (yield Wait(self.o_full[s], (j >> 1) - 1, 0x609)):
                self.abort = True
                break
            self.begin(agent, f"V{s}", "r")
            self.check(agent, f"V{s}", j)
            self.begin(agent, f"VT{s}.{w}", "w")
            self.mem[f"VT{s}.{w}"] = j
            yield None
            self.end(agent, f"VT{s}.{w}", "w")
            self.vt_full[s].arrive(32)
            if self.named:
                self.end(agent, f"V{s}", "r")
                yield NamedWait(self.tr_bar)
                if w == 0:
                    self.kv_empty[s].arrive()
            else:
                self.end(agent, f"V{s}", "r")
                self.kv_empty[s].arrive()
            yield None

    def softmax(self, w):
        agent = f"softmax{w}"
        ok = True
        for j in range(self.n_kb):
            s = j & 1
            if not (yield Wait(self.s_full[s], j >> 1, 0x60a)):
                ok = False
                break
            self.begin(agent, f"S{s}.{w}", "r")
            self.check(agent, f"S{s}.{w}", j)
            yield None
            self.end(agent, f"S{s}.{w}", "r")
            self.s_free[s].arrive(32)
            self.begin(agent, f"P{s}.{w}", "w")
            self.mem[f"P{s}.{w}"] = j
            yield None
            self.end(agent, f"P{s}.{w}", "w")
            self.p_full[s].arrive(32)
            if not (yield Wait(self.o_full[s], j >> 1, 0x60b)):
                ok = False
                break
            self.begin(agent, f"O{s}.{w}", "r")
            self.check(agent, f"O{s}.{w}", j)
            yield None
            self.end(agent, f"O{s}.{w}", "r")
            self.o_free[s].arrive(32)
            self.seen[w].append(j)
        if not ok:
            self.abort = True

    # ------------------------------------------------------------ scheduler
    def roles(self) -> dict:
        roles = {"producer": self.producer(), "mma": self.mma_issuer()}
        for w in range(2):
            roles[f"transposer{w}"] = self.transposer(w)
        for w in range(4):
            roles[f"softmax{w}"] = self.softmax(w)
        return roles

    def run(self, max_steps: int = 200000) -> str:
        """Returns "done" or "deadlock" (roles blocked on a barrier without a
        time limit).  Errors are collected in self.errors."""
        roles = self.roles()
        pending = {}
        for name, g in roles.items():
            pending[name] = self._advance(g, None, name)
        pending = {k: v for k, v in pending.items() if v != "exit"}
        faulted = self.fault_at is None
        steps = 0
        while pending and steps < max_steps:
            steps += 1
            for n, w in pending.items():
                if isinstance(w, Wait):
                    h = w.hazard()
                    if h and h not in self.errors:
                        self.errors.append(f"{n} {h}")
            runnable = [n for n, w in pending.items() if w is None or w.ready()]
            asyncs = [("tma", i) for i in range(len(self.tma))] + ([("pipe", 0)] if self.pipe else [])
            timed = [n for n, w in pending.items()
                     if isinstance(w, Wait) and not w.ready() and w.code is not None]
            if not faulted and steps >= self.fault_at and timed:
                faulted = True
                name = self.rng.choice(timed)
                self._give_up(pending[name])
                pending[name] = self._advance(roles[name], False, name)
                if pending[name] == "exit":
                    del pending[name]
                continue
            choices = [("role", n) for n in runnable] + asyncs
            if not choices:
                blocked = [n for n, w in pending.items() if isinstance(w, Wait)]
                if not blocked:
                    return "deadlock"
                name = self.rng.choice(blocked)    # a bounded wait runs out
                self._give_up(pending[name])
                pending[name] = self._advance(roles[name], False, name)
                if pending[name] == "exit":
                    del pending[name]
                continue
            kind, x = self.rng.choice(choices)
            if kind == "tma":
                self._complete_tma(x)
            elif kind == "pipe":
                self._complete_pipe()
            else:
                w = pending[x]
                val = None
                if w is not None:
                    val = True
                    if isinstance(w, Wait) and w.bar.phase != w.phase + 1:
                        self.errors.append(f"{x} waited for phase {w.phase} of {w.bar.name}, "
                                           f"which is at {w.bar.phase} (lapped)")
                pending[x] = self._advance(roles[x], val, x)
                if pending[x] == "exit":
                    del pending[x]
        if pending:
            return "deadlock"
        # the CTA's exit: TMEM is freed and shared memory released
        if self.tma:
            self.errors.append(f"{len(self.tma)} TMA loads still in flight at exit")
        if self.pipe:
            self.errors.append(f"{len(self.pipe)} tensor-core operations still queued at exit")
        return "done"

    def _give_up(self, w: Wait):
        if w.code is not None and self.err == 0:
            self.err = w.code

    @staticmethod
    def _advance(gen, value, name):
        try:
            return gen.send(value) if value is not None else next(gen)
        except StopIteration:
            return "exit"


class ModelMN(Model):
    """Variant 1 of the kernel (attn_prefill_tc_mn_kernel): no transposers; V
    feeds the O MMA in place; O accumulates in TMEM across tiles (each O MMA
    reads the previous tile's O and writes its own); kv_empty takes one commit
    after O_j; o_full[s] counts the O MMAs of tiles with parity s; a softmax
    warp that moves its base (drawn at random here, `rescale_p`) waits for
    O_{j-1} and rewrites its quarter of O before releasing P_j.  Softmax waits
    are warp-uniform in the kernel, so one warp is one role."""

    def __init__(self, n_kb: int, seed: int, fault_at=None, rescale_p: float = 0.3):
        super().__init__(n_kb, seed, fault_at)
        self.kv_empty = [Bar(f"kv_empty{i}", 1) for i in range(2)]
        self.rescale_p = rescale_p
        self.rescales = 0

    def roles(self) -> dict:
        roles = {"producer": self.producer(), "mma": self.mma_issuer()}
        for w in range(4):
            roles[f"softmax{w}"] = self.softmax(w)
        return roles

    def producer(self):
        n_kb = self.n_kb
        self.q_full.arrive_expect_tx(Q_BYTES)
        self.tma_load("Q", self.q_full, Q_BYTES, "q")
        yield None
        issued = 0
        for j in range(n_kb):
            if self.abort:
                break
            s = j & 1
            if j >= 2 and not (yield Wait(self.kv_empty[s], (j >> 1) - 1, 0x611)):
                self.abort = True
                break
            self.kv_full[s].arrive_expect_tx(2 * KV_BYTES)
            self.tma_load(f"K{s}", self.kv_full[s], KV_BYTES, j)
            self.tma_load(f"V{s}", self.kv_full[s], KV_BYTES, j)
            issued = j + 1
            yield None
        yield Wait(self.q_full, 0, None)
        for j in range(max(0, issued - 2), issued):
            yield Wait(self.kv_full[j & 1], j >> 1, None)

    def mma_issuer(self):
        n_kb = self.n_kb
        ok = yield Wait(self.q_full, 0, 0x612)

        def issue_s(j):
            s = j & 1
            if not (yield Wait(self.kv_full[s], j >> 1, 0x613)):
                return False
            self.mma([("Q", "q"), (f"K{s}", j)], [(f"S{s}.{w}", j) for w in range(4)])
            self.commit(self.s_full[s])
            return True

        if ok and n_kb > 0:
            ok = yield from issue_s(0)
        j = 0
        while ok and j < n_kb and not self.abort:
            if j + 1 < n_kb and not (yield from issue_s(j + 1)):
                ok = False
                break
            s = j & 1
            if not (yield Wait(self.p_full[s], j >> 1, 0x614)):
                ok = False
                break
            reads = [(f"P{s}.{w}", j) for w in range(4)] + [(f"V{s}", j)]
            if j > 0:
                reads += [(f"O.{w}", j - 1) for w in range(4)]
            self.mma(reads, [(f"O.{w}", j) for w in range(4)])
            self.commit(self.o_full[s])
            self.commit(self.kv_empty[s])
            j += 1
            yield None
        if not ok:
            self.abort = True
        self.commit(self.mma_done)
        yield Wait(self.mma_done, 0, None)

    def transposer(self, w):      # not in this variant
        return iter(())

    def softmax(self, w):
        agent = f"softmax{w}"
        n_kb = self.n_kb
        ok = True
        for j in range(n_kb):
            if self.abort:
                break
            s = j & 1
            if not (yield Wait(self.s_full[s], j >> 1, 0x615)):
                ok = False
                break
            self.begin(agent, f"S{s}.{w}", "r")
            self.check(agent, f"S{s}.{w}", j)
            yield None
            self.end(agent, f"S{s}.{w}", "r")
            if j >= 2 and not (yield Wait(self.o_full[s], (j >> 1) - 1, 0x616)):
                ok = False
                break
            if j > 0 and self.rng.random() < self.rescale_p:
                if not (yield Wait(self.o_full[(j - 1) & 1], (j - 1) >> 1, 0x617)):
                    ok = False
                    break
                self.rescales += 1
                self.begin(agent, f"O.{w}", "w")
                self.check(agent, f"O.{w}", j - 1)
                yield None
                self.end(agent, f"O.{w}", "w")
            self.begin(agent, f"P{s}.{w}", "w")
            self.mem[f"P{s}.{w}"] = j
            yield None
            self.end(agent, f"P{s}.{w}", "w")
            self.p_full[s].arrive(32)
        if not ok:
            self.abort = True
        if ok and not self.abort and n_kb > 0:
            last = n_kb - 1
            if (yield Wait(self.o_full[last & 1], last >> 1, 0x618)):
                self.begin(agent, f"O.{w}", "r")
                self.check(agent, f"O.{w}", last)
                yield None
                self.end(agent, f"O.{w}", "r")
                self.seen[w] = list(range(n_kb))


class ModelPP(Model):
    """Variant 2 of the kernel (attn_prefill_tc_pp_kernel): persistent, two
    query tiles (two heads of one KV head) per item, 128-key tiles.  `items`
    lists the key-tile count of each item this CTA runs in order (n_kb alone
    is one item).  K and V have their own 2-deep rings (k_empty after S_j of
    both tiles, v_empty after PV_j of both); the MMA thread alternates
    PV_j(0), S_{j+1}(0), PV_j(1), S_{j+1}(1); P_j(t) overwrites S[t] in TMEM
    (same buffer here, tagged ("p", item, j)), so the next S MMA of the tile
    runs only after the PV that reads it (program order on the tensor pipe);
    O[t] accumulates in TMEM and a softmax warp may rescale its quarter once it
    has seen S_j(t) (the commit of S_j(t) covers PV_{j-1}(t)).  Across items:
    the producer reloads Q after q_empty (the item's last S MMAs), and an
    item's first PV overwrites O[t] only after every softmax warp of the tile
    read out the previous item's O[t] (o_empty).  One role per softmax warp:
    warps 2-5 hold tile 0, warps 6-9 tile 1."""

    KV128 = 128 * 128 * 2

    def __init__(self, n_kb: int, seed: int, fault_at=None, rescale_p: float = 0.3, items=None):
        super().__init__(n_kb, seed, fault_at)
        self.items = list(items) if items is not None else [n_kb]
        self.k_full = [Bar(f"k_full{i}", 1) for i in range(2)]
        self.k_empty = [Bar(f"k_empty{i}", 1) for i in range(2)]
        self.v_full = [Bar(f"v_full{i}", 1) for i in range(2)]
        self.v_empty = [Bar(f"v_empty{i}", 1) for i in range(2)]
        self.s_full = [Bar(f"s_full{t}", 1) for t in range(2)]
        self.p_full = [Bar(f"p_full{t}", 4) for t in range(2)]
        self.o_final = [Bar(f"o_final{t}", 1) for t in range(2)]
        self.o_empty = [Bar(f"o_empty{t}", 4) for t in range(2)]
        self.q_empty = Bar("q_empty", 1)
        self.rescale_p = rescale_p
        self.rescales = 0

    def roles(self) -> dict:
        roles = {"producer": self.producer(), "mma": self.mma_issuer()}
        for t in range(2):
            for w in range(4):
                roles[f"softmax{t}.{w}"] = self.softmax(t, w)
        return roles

    def producer(self):
        KV = self.KV128
        T = ic = nk = nv = 0
        ok = True
        for it, n_kb in enumerate(self.items):
            if not ok or self.abort:
                break
            if ic >= 1 and not (yield Wait(self.q_empty, ic - 1, 0x63b)):
                ok = False
                break
            self.q_full.arrive_expect_tx(2 * Q_BYTES)
            self.tma_load("Q0", self.q_full, Q_BYTES, ("q", it))
            self.tma_load("Q1", self.q_full, Q_BYTES, ("q", it))
            ic += 1
            yield None
            for j in range(n_kb):
                s = T & 1
                if T >= 2 and not (yield Wait(self.k_empty[s], (T >> 1) - 1, 0x631)):
                    ok = False
                    break
                self.k_full[s].arrive_expect_tx(KV)
                self.tma_load(f"K{s}", self.k_full[s], KV, (it, j))
                nk = T + 1
                if T >= 2 and not (yield Wait(self.v_empty[s], (T >> 1) - 1, 0x632)):
                    ok = False
                    break
                self.v_full[s].arrive_expect_tx(KV)
                self.tma_load(f"V{s}", self.v_full[s], KV, (it, j))
                nv = T + 1
                T += 1
                yield None
        if not ok:
            self.abort = True
        if ic > 0:
            yield Wait(self.q_full, ic - 1, None)
        for j in range(max(0, nk - 2), nk):
            yield Wait(self.k_full[j & 1], j >> 1, None)
        for j in range(max(0, nv - 2), nv):
            yield Wait(self.v_full[j & 1], j >> 1, None)

    def mma_issuer(self):
        def issue_s(it, j, T, t):
            self.mma([(f"Q{t}", ("q", it)), (f"K{T & 1}", (it, j))],
                     [(f"S{t}.{w}", ("s", it, j)) for w in range(4)])
            self.commit(self.s_full[t])

        def issue_pv(it, j, T, t):
            reads = [(f"S{t}.{w}", ("p", it, j)) for w in range(4)] + [(f"V{T & 1}", (it, j))]
            if j > 0:
                reads += [(f"O{t}.{w}", (it, j - 1)) for w in range(4)]
            self.mma(reads, [(f"O{t}.{w}", (it, j)) for w in range(4)])

        ok = True
        T = ic = 0
        for it, n_kb in enumerate(self.items):
            if not ok or self.abort:
                break
            if not (yield Wait(self.q_full, ic, 0x633)) or \
                    not (yield Wait(self.k_full[T & 1], T >> 1, 0x634)):
                ok = False
                break
            issue_s(it, 0, T, 0)
            issue_s(it, 0, T, 1)
            self.commit(self.k_empty[T & 1])
            if n_kb == 1:
                self.commit(self.q_empty)
            for j in range(n_kb):
                Tj = T + j
                if not (yield Wait(self.v_full[Tj & 1], Tj >> 1, 0x635)):
                    ok = False
                    break
                for t in range(2):
                    if not (yield Wait(self.p_full[t], Tj, 0x636)):
                        ok = False
                        break
                    if j == 0 and ic >= 1 and not (yield Wait(self.o_empty[t], ic - 1, 0x63c)):
                        ok = False
                        break
                    issue_pv(it, j, Tj, t)
                    if t == 1:
                        self.commit(self.v_empty[Tj & 1])
                    if j + 1 < n_kb:
                        if t == 0 and not (yield Wait(self.k_full[(Tj + 1) & 1], (Tj + 1) >> 1,
                                                      0x637)):
                            ok = False
                            break
                        issue_s(it, j + 1, Tj + 1, t)
                        if t == 1:
                            self.commit(self.k_empty[(Tj + 1) & 1])
                            if j + 2 == n_kb:
                                self.commit(self.q_empty)
                    else:
                        self.commit(self.o_final[t])
                    yield None
                if not ok:
                    break
            T += n_kb
            ic += 1
        if not ok:
            self.abort = True
        self.commit(self.mma_done)
        yield Wait(self.mma_done, 0, None)

    def softmax(self, t, w):
        agent = f"softmax{t}.{w}"
        ok = True
        T = ic = 0
        for it, n_kb in enumerate(self.items):
            for j in range(n_kb):
                Tj = T + j
                if self.abort:
                    ok = False
                    break
                if not (yield Wait(self.s_full[t], Tj, 0x638)):
                    ok = False
                    break
                buf = f"S{t}.{w}"
                self.begin(agent, buf, "r")
                self.check(agent, buf, ("s", it, j))
                yield None
                self.end(agent, buf, "r")
                self.begin(agent, buf, "w")            # P_j over S_j
                self.mem[buf] = ("p", it, j)
                yield None
                self.end(agent, buf, "w")
                if j > 0 and self.rng.random() < self.rescale_p:
                    self.rescales += 1
                    self.begin(agent, f"O{t}.{w}", "w")
                    self.check(agent, f"O{t}.{w}", (it, j - 1))
                    yield None
                    self.end(agent, f"O{t}.{w}", "w")
                self.p_full[t].arrive()
            if not ok:
                break
            if not (yield Wait(self.o_final[t], ic, 0x639)):
                ok = False
                break
            self.begin(agent, f"O{t}.{w}", "r")
            self.check(agent, f"O{t}.{w}", (it, n_kb - 1))
            yield None
            self.end(agent, f"O{t}.{w}", "r")
            self.o_empty[t].arrive()
            self.seen[(t, w)].append(it)
            T += n_kb
            ic += 1
        if not ok:
            self.abort = True
