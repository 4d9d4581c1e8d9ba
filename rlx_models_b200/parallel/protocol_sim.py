"""Host emulation of the device flag protocols of the NVLink collectives.

The peer-memory kernels (``csrc/comm/tp_fused.cu`` ``ar_pull_norm`` /
``ar2_norm``, ``csrc/comm/tp_sample.cu`` ``tp_argmax``) synchronise ranks with
epoch flags (or, for the argmax, keys that carry their op's tag) and reuse
their buffers without host involvement. Their
correctness rests on ordering arguments ("a rank rewrites this slot only after
every peer passed the next barrier, which it does after finishing its reads").
This module replays each protocol step by step on the host:

* every rank is a stream of kernels; a kernel's CTAs become runnable when the
  rank's previous kernel has finished completely (stream order, as the
  kernels' ``griddepcontrol.wait`` enforces under programmatic launch);
* CTAs are generators; a scheduler with a seeded RNG picks which runnable CTA
  of which rank advances next, so many seeds cover many interleavings of CTAs
  across and within ranks;
* shared memory holds *tags* (which op wrote a value) instead of numbers, and
  every read asserts that it sees the tag of the op it belongs to: a stale
  read, a read of a slot already overwritten by a later op, or a write into a
  slot someone may still read fails immediately, naming the op and rank.

A protocol that can deadlock leaves no runnable CTA before the streams
finish; the scheduler reports that as well. The model is sequentially
consistent; on the GPU the release / acquire flag operations and the
system-scope fences provide the orderings the model assumes.

Reference: no counterpart in the reference (its collectives are host
driven); the plan for comm-kernel race detection asks for host emulation of
the protocols over CPU ranks.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field

ZERO = "zero"


class ProtocolError(AssertionError):
    pass


@dataclass
class Wait:
    """Yielded by a CTA: block until ``pred()`` holds."""
    pred: object


@dataclass
class Rank:
    idx: int
    mem: dict = field(default_factory=dict)
    kernels: list = field(default_factory=list)   # [(name, [cta factories])]
    running: list = field(default_factory=list)   # live CTA generators of the current kernel
    pending: list = field(default_factory=list)   # (gen, Wait) blocked CTAs


class Sim:
    def __init__(self, world: int, seed: int = 0):
        self.world = world
        self.rng = random.Random(seed)
        self.ranks = [Rank(i) for i in range(world)]
        self.steps = 0

    def mem(self, rank: int) -> dict:
        return self.ranks[rank].mem

    def launch(self, rank: int, name: str, ctas: list):
        """Queue a kernel (a list of CTA generator factories) on ``rank``'s stream."""
        self.ranks[rank].kernels.append((name, ctas))

    def _start_next(self, r: Rank):
        if not r.running and not r.pending and r.kernels:
            _, ctas = r.kernels.pop(0)
            r.running = [f() for f in ctas]

    def run(self, max_steps: int = 2_000_000):
        for r in self.ranks:
            self._start_next(r)
        while True:
            # wake blocked CTAs whose condition holds
            for r in self.ranks:
                still = []
                for gen, w in r.pending:
                    if w.pred():
                        r.running.append(gen)
                    else:
                        still.append((gen, w))
                r.pending = still
            live = [(r, g) for r in self.ranks for g in r.running]
            if not live:
                if any(r.pending or r.kernels for r in self.ranks):
                    blocked = {r.idx: len(r.pending) for r in self.ranks if r.pending}
                    raise ProtocolError(f"deadlock: no runnable CTA, blocked per rank {blocked}")
                return self.steps
            r, g = live[self.rng.randrange(len(live))]
            self.steps += 1
            if self.steps > max_steps:
                raise ProtocolError("step budget exhausted")
            try:
                y = next(g)
            except StopIteration:
                r.running.remove(g)
                self._start_next(r)
                continue
            if isinstance(y, Wait) and not y.pred():
                r.running.remove(g)
                r.pending.append((g, y))


def _check(cond: bool, msg: str):
    if not cond:
        raise ProtocolError(msg)


# ---------------------------------------------------------------------------
# tensor-parallel decode all-reduce (+ residual add + RMSNorm)
# ---------------------------------------------------------------------------

def setup_tp(sim: Sim, rows: int):
    """Symmetric buffers of the pull communicator: fp32 partial slots by
    parity, one-shot flags, two-shot result slots and flags, local counters."""
    W = sim.world
    rpr_max = -(-rows // W)
    for q in range(W):
        m = sim.mem(q)
        m["acc"] = [[ZERO] * rows for _ in range(2)]
        m["flags"] = [0] * W
        m["res"] = {}  # (owned row, slice) -> op that wrote it
        m["flags2"] = [[0] * W for _ in range(2)]
        m["out"] = [None] * rows
        m["ctr1"] = dict(epoch=0, dep=0)
        m["ctr2"] = dict(epoch=0, arr=0, dep=0)


def gemm_acc(sim: Sim, rank: int, op: int, par: int, M: int):
    """The accumulate-mode GEMM of op ``op``: adds into acc[par], which must be clear."""
    def cta(row):
        def g():
            m = sim.mem(rank)
            _check(m["acc"][par][row] == ZERO,
                   f"rank {rank} op {op}: GEMM accumulates into acc[{par}][{row}] still holding {m['acc'][par][row]}")
            yield
            m["acc"][par][row] = op
        return g
    sim.launch(rank, f"gemm{op}", [cta(r) for r in range(M)])


def ar_pull(sim: Sim, rank: int, op: int, par: int, M: int, rows: int):
    """ar_pull_norm_kernel: one barrier, every rank reads every row of every partial."""
    W = sim.world
    grid = max(M, rows)

    def cta(i):
        def g():
            m = sim.mem(rank)
            e = m["ctr1"]["epoch"] + 1
            if i == 0:
                for q in range(W):
                    sim.mem(q)["flags"][rank] = e
                    yield
            yield Wait(lambda: all(f >= e for f in m["flags"]))
            if i < M:
                for q in range(W):
                    v = sim.mem(q)["acc"][par][i]
                    _check(v == op, f"rank {rank} op {op}: pulled rank {q} acc[{par}][{i}] = {v}")
                    yield
                m["out"][i] = op
            if i < rows:
                m["acc"][par ^ 1][i] = ZERO
            yield
            m["ctr1"]["dep"] += 1
            if m["ctr1"]["dep"] == grid:
                m["ctr1"]["dep"] = 0
                m["ctr1"]["epoch"] = e
        return g
    sim.launch(rank, f"pull{op}", [cta(i) for i in range(grid)])


def ar2(sim: Sim, rank: int, op: int, par: int, M: int, rows: int, slices: int = 2):
    """ar2_norm_kernel: (owned row, column slice) items reduced after barrier 1 by
    CTAs i, i + grid, ...; every row (residual slices + slice sums of squares)
    copied from its owner by everyone after barrier 2."""
    W = sim.world
    rpr = -(-M // W)
    n_my = max(0, min(rpr, M - rank * rpr))
    n_items = n_my * slices
    grid = max(M, rows)

    def cta(i):
        def g():
            m = sim.mem(rank)
            e = m["ctr2"]["epoch"] + 1
            if i == 0:
                for q in range(W):
                    sim.mem(q)["flags2"][0][rank] = e
                    yield
            if i < n_items:
                yield Wait(lambda: all(f >= e for f in m["flags2"][0]))
                for item in range(i, n_items, grid):
                    li, sl = divmod(item, slices)
                    row = rank * rpr + li
                    for q in range(W):
                        v = sim.mem(q)["acc"][par][row]
                        _check(v == op, f"rank {rank} op {op}: reduced rank {q} acc[{par}][{row}] = {v}")
                        yield
                    m["res"][(li, sl)] = op
                    yield
                    m["ctr2"]["arr"] += 1
                    if m["ctr2"]["arr"] == n_items:
                        for q in range(W):
                            sim.mem(q)["flags2"][1][rank] = e
                            yield
            elif n_my == 0 and i == 0:
                for q in range(W):
                    sim.mem(q)["flags2"][1][rank] = e
                    yield
            yield Wait(lambda: all(f >= e for f in m["flags2"][1]))
            if i < M:
                owner, j = i // rpr, i % rpr
                for sl in range(slices):
                    v = sim.mem(owner)["res"].get((j, sl))
                    _check(v == op, f"rank {rank} op {op}: copied row {i} slice {sl} from rank {owner} = {v}")
                    yield
                m["out"][i] = op
            if i < rows:
                m["acc"][par ^ 1][i] = ZERO
            yield
            m["ctr2"]["dep"] += 1
            if m["ctr2"]["dep"] == grid:
                m["ctr2"]["arr"] = 0
                m["ctr2"]["dep"] = 0
                m["ctr2"]["epoch"] = e
        return g
    sim.launch(rank, f"ar2_{op}", [cta(i) for i in range(grid)])


def tp_decode_ops(world: int, M: int, n_ops: int, seed: int, rows: int = 8, mode: str = "mixed") -> int:
    """``n_ops`` row-parallel ops (GEMM into acc[parity] + reduction kernel) on
    every rank; ``mode`` "pull", "two_shot" or "mixed" (a per-op choice, the
    same on every rank, as the communicator makes it from M). Returns the
    number of scheduler steps taken."""
    sim = Sim(world, seed)
    setup_tp(sim, rows)
    pick = random.Random(seed + 1)
    kinds = [("two_shot" if mode == "two_shot" else "pull" if mode == "pull" else pick.choice(["pull", "two_shot"]))
             for _ in range(n_ops)]
    for op in range(1, n_ops + 1):
        par = op & 1
        for r in range(world):
            gemm_acc(sim, r, op, par, M)
            (ar2 if kinds[op - 1] == "two_shot" else ar_pull)(sim, r, op, par, M, rows)
    return sim.run()


# ---------------------------------------------------------------------------
# vocab-parallel greedy argmax
# ---------------------------------------------------------------------------

def tp_argmax_ops(world: int, R: int, n_ops: int, seed: int, buffers: int = 2) -> int:
    """``tp_argmax_kernel``: every rank pushes row r's tagged key into slot
    [parity][r][rank] of every rank, then polls its own slots [parity][r][q]
    until each holds a key, reads and clears them. A writer must never find an
    unread key in a slot, and a reader must only ever find this op's key.
    ``buffers=1`` models a single-buffered variant (for the negative test)."""
    sim = Sim(world, seed)
    for q in range(world):
        m = sim.mem(q)
        m["keys"] = [[[None] * world for _ in range(R)] for _ in range(2)]
        m["ctr"] = dict(epoch=0, dep=0)

    def kernel(rank, op):
        def cta(row):
            def g():
                m = sim.mem(rank)
                e = m["ctr"]["epoch"] + 1
                par = e % buffers
                _check(e == op, f"rank {rank}: epoch {e} for op {op}")
                for q in range(world):
                    slot = sim.mem(q)["keys"][par][row]
                    _check(slot[rank] is None,
                           f"rank {rank} op {op}: rank {q} slot [{par}][{row}][{rank}] still holds op {slot[rank]}")
                    slot[rank] = op
                    yield
                for q in range(world):
                    yield Wait(lambda q=q: m["keys"][par][row][q] is not None)
                    v = m["keys"][par][row][q]
                    _check(v == op, f"rank {rank} op {op}: slot [{par}][{row}][{q}] holds op {v}")
                    m["keys"][par][row][q] = None
                    yield
                m["ctr"]["dep"] += 1
                if m["ctr"]["dep"] == R:
                    m["ctr"]["dep"] = 0
                    m["ctr"]["epoch"] = e
            return g
        return [cta(r) for r in range(R)]

    for op in range(1, n_ops + 1):
        for r in range(world):
            sim.launch(r, f"argmax{op}", kernel(r, op))
    return sim.run()
