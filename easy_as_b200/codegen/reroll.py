"""Find Python-unrolled loops in straight-line IR so the emitter can print them as loops.

DSL kernels unroll ``for`` loops at trace time: the tracer runs the Python
function once, so a loop over a constexpr range leaves one copy of its body
per iteration in the IR (easy_as ``eas/compiler.py:553-601``).  Kernels such
as the tiled matmul at K = 2048 then have thousands of instructions, which
makes NVRTC slow and the cubin large.

A *run* is ``count >= 3`` consecutive blocks of ``length`` instructions of the
instruction stream (``arg``, ``const`` and ``alloc_tg`` excluded: the thread
emitter prints them before the body) in which instruction ``j`` of every
block has the same op, output type and literal operands, and each value
operand of block ``r`` is, position by position,

* ``("local", q)``: the value of instruction ``q`` of the same block;
* ``("carry", q, init)``: the value of instruction ``q`` of block ``r - 1``,
  and in block 0 the value ``init`` defined before the run;
* ``("inv", id)``: the same value, defined before the run, in every block;
* ``("affine", c0, d)``: a u32 constant equal to ``c0 + r*d`` (mod 2^32).

Only values of the last block may be read after the run.  Printing block 0
inside ``for (r = 0; r < count; ++r)`` with those substitutions performs the
same operations in the same order as the unrolled code, so results are
bit-identical.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from ..ir import DType, Inst, ValueRef

SKIP = frozenset({"arg", "const", "alloc_tg"})


@dataclass(frozen=True)
class Run:
    first: tuple[int, ...]                  # IR indices of block 0's instructions
    stream_start: int                       # position of block 0 in the instruction stream
    ir_span: frozenset[int]                 # IR indices of every instruction of the run
    blocks: tuple[tuple[int, ...], ...]     # IR indices per block
    length: int
    count: int
    forms: tuple[tuple[Any, ...], ...]      # per block-0 instruction: one form per operand
    escapes: tuple[int, ...]                # q whose last-block value is read after the run
    last_out: tuple[int | None, ...]        # per q: value id made by the last block (None: no output)


def _token(i: Inst) -> tuple[Any, ...]:
    out = None if i.out is None else (i.out.dtype, i.out.lanes)
    lits = tuple((None if isinstance(a, ValueRef) else a) for a in i.args)
    return (i.op, out, lits)


class _Finder:
    def __init__(self, insts: tuple[Inst, ...]):
        self.insts = insts
        self.pos = [k for k, i in enumerate(insts) if i.op not in SKIP]
        self.toks = [_token(insts[k]) for k in self.pos]
        self.u32 = {i.out.id: int(i.args[0]) for i in insts
                    if i.op == "const" and i.out is not None and i.out.dtype == DType.U32
                    and not isinstance(i.args[0], bool)}
        self.defpos: dict[int, int] = {}
        for k, i in enumerate(insts):
            if i.out is not None:
                self.defpos[i.out.id] = k
        self.users: dict[int, list[int]] = {}
        for k, i in enumerate(insts):
            for a in i.args:
                if isinstance(a, ValueRef):
                    self.users.setdefault(a.id, []).append(k)

    def candidates(self) -> list[int]:
        anchors: dict[Any, list[int]] = {}
        for s, t in enumerate(self.toks):
            if t[0] in ("barrier", "dot", "store", "mma", "load", "mma_store"):
                anchors.setdefault(t, []).append(s)
        cands: set[int] = set()
        for occ in anchors.values():
            for a in range(len(occ) - 1):
                for b in range(a + 1, min(len(occ), a + 5)):
                    g = occ[b] - occ[a]
                    if 2 <= g <= 4096:
                        cands.add(g)
        return sorted(cands)

    def scan(self, L: int, min_count: int, min_saved: int, keep: tuple[frozenset[int], ...]) -> list[Run]:
        """Runs of one period, left to right, non-overlapping.  Where a stretch of repeats starts
        at a phase that splits a ``keep`` group, the later phases of the stretch are tried."""
        toks, n = self.toks, len(self.toks)
        out: list[Run] = []
        s = 0
        while s + 2 * L < n:
            if toks[s] != toks[s + L]:
                s += 1
                continue
            e = s
            while e + L < n and toks[e] == toks[e + L]:
                e += 1
            run = None
            for p in range(s, min(s + L, e)):
                count = (e - p) // L + 1
                if count < min_count or (count - 1) * L < min_saved:
                    break
                got = self.verify(p, L, count)
                if got is None or got < min_count or (got - 1) * L < min_saved:
                    continue
                run = self.build(p, L, got)
                if run is not None and _respects(run, keep):
                    break
                run = None
            if run is not None:
                out.append(run)
                s = run.stream_start + L * run.count
            else:
                s = e + 1
        return out

    def _form(self, where: dict[int, tuple[int, int]], r: int, a: Any) -> tuple[Any, ...]:
        if not isinstance(a, ValueRef):
            return ("lit",)
        w = where.get(a.id)
        if w is None:
            return ("const", self.u32[a.id]) if a.id in self.u32 else ("ext", a.id)
        br, q = w
        if br == r:
            return ("local", q)
        if br == r - 1:
            return ("carry", q)
        return ("far",)

    def verify(self, s: int, L: int, count: int) -> int | None:
        """Number of leading blocks (from the candidate start) that form a run, or None."""
        insts, pos = self.insts, self.pos
        where: dict[int, tuple[int, int]] = {}
        for r in range(count):
            for j in range(L):
                o = insts[pos[s + r * L + j]].out
                if o is not None:
                    where[o.id] = (r, j)
        f0 = [[self._form(where, 0, a) for a in insts[pos[s + j]].args] for j in range(L)]
        if any(f[0] in ("far", "carry") for fs in f0 for f in fs):
            return None
        deltas: dict[tuple[int, int], int] = {}
        carried: dict[tuple[int, int], int] = {}
        good = 1
        for r in range(1, count):
            for j in range(L):
                for k, a in enumerate(insts[pos[s + r * L + j]].args):
                    a0, fr = f0[j][k], self._form(where, r, a)
                    if a0[0] == "const" and fr[0] == "const":
                        d = (fr[1] - a0[1]) % (1 << 32)
                        if r == 1:
                            deltas[(j, k)] = d
                        if (deltas[(j, k)] * r - d) % (1 << 32) == 0:
                            continue
                        return good if good >= 3 else None
                    if a0[0] == "ext" and fr[0] == "carry":
                        if carried.setdefault((j, k), fr[1]) == fr[1]:
                            continue
                        return good if good >= 3 else None
                    if a0 == fr and a0[0] in ("lit", "local", "ext"):
                        continue
                    return good if good >= 3 else None
            good = r + 1
        return good

    def build(self, s: int, L: int, count: int) -> Run | None:
        insts, pos = self.insts, self.pos
        blocks = [[pos[s + r * L + j] for j in range(L)] for r in range(count)]
        span = frozenset(k for b in blocks for k in b)
        where: dict[int, tuple[int, int]] = {}
        for r, b in enumerate(blocks):
            for j, k in enumerate(b):
                o = insts[k].out
                if o is not None:
                    where[o.id] = (r, j)
        forms = []
        for j, k in enumerate(blocks[0]):
            fj = []
            for kk, a in enumerate(insts[k].args):
                if not isinstance(a, ValueRef):
                    fj.append(("lit",))
                    continue
                w = where.get(a.id)
                if w is not None:
                    fj.append(("local", w[1]))
                    continue
                a1 = insts[blocks[1][j]].args[kk]
                w1 = where.get(a1.id)
                if w1 is not None:  # block 1 reads block 0: carried
                    fj.append(("carry", w1[1], a.id))
                elif a.id in self.u32 and a1.id != a.id:
                    d = (self.u32[a1.id] - self.u32[a.id]) % (1 << 32)
                    fj.append(("affine", self.u32[a.id], d))
                else:
                    fj.append(("inv", a.id))
            forms.append(tuple(fj))
        # only the last block's values may be read outside the run
        escapes = []
        for r, b in enumerate(blocks):
            for j, k in enumerate(b):
                o = insts[k].out
                if o is None:
                    continue
                outside = [u for u in self.users.get(o.id, ()) if u not in span]
                if outside and r != count - 1:
                    return None
                if outside:
                    escapes.append(j)
        last = tuple(None if insts[k].out is None else insts[k].out.id for k in blocks[-1])
        return Run(first=tuple(blocks[0]), stream_start=s, ir_span=span,
                   blocks=tuple(tuple(b) for b in blocks), length=L, count=count, forms=tuple(forms),
                   escapes=tuple(escapes), last_out=last)


def find_runs(insts: tuple[Inst, ...], *, min_count: int = 3, min_saved: int = 24,
              keep_together: tuple[frozenset[int], ...] = ()) -> list[Run]:
    """Non-overlapping runs, largest coverage first.  ``keep_together``: sets of IR indices that
    must fall in one block of a run, or outside all runs (e.g. dots the emitter fuses)."""
    f = _Finder(insts)
    found: list[Run] = []
    for L in f.candidates():
        found += f.scan(L, min_count, min_saved, keep_together)
    found.sort(key=lambda r: (-(r.length * (r.count - 1)), r.length, r.stream_start))
    taken = [False] * len(f.pos)
    runs: list[Run] = []
    for run in found:
        lo, hi = run.stream_start, run.stream_start + run.length * run.count
        if any(taken[lo:hi]):
            continue
        for x in range(lo, hi):
            taken[x] = True
        runs.append(run)
    runs.sort(key=lambda r: r.first[0])
    return runs


def _respects(run: Run, groups: tuple[frozenset[int], ...]) -> bool:
    """Every group lies within one block of the run or wholly outside it."""
    block_of = {k: r for r, b in enumerate(run.blocks) for k in b}
    for g in groups:
        where = {block_of.get(k) for k in g}
        if len(where) > 1:
            return False
    return True
