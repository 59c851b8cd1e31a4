"""Prove that a thread-mode kernel is a (masked, tiled) fp32 GEMM, and launch the native FFMA kernel for it.

Targets: the reference's fp32 matmul kernels (easy_as ``examples/matmul_tiled.py:27-230``, the
masked ``matmul_tiled_kernel`` and the interior ``matmul_tiled_full_kernel``, and the naive
``examples/matmul.py:23-43``).  The tiled ones copy A and B tiles into threadgroup memory, sync,
run ``mk.dot`` over the tiles and add each dot to a running sum; the naive one is one ``fma``
chain per output.  The generic lowering keeps their thread structure, so it is bound by
shared-memory or L1 reads.

Nothing here matches source text or instruction order.  For a given launch (scalar argument
values, grid, threads per group) the whole thread group is executed symbolically, all threads at
once:

* every u32 value is, per thread, a linear form ``c + a0*P0 + a1*P1 + a2*P2`` modulo 2^32 in the
  program ids (numpy arrays over the threads); products, divisions and remainders need an operand
  free of the program ids, so the forms stay linear and the divisions exact;
* a mask is a per-thread boolean (the comparisons between program-id-free values) and a list of
  atoms ``lhs < rhs`` whose left side depends on the program ids;
* a float value is a term: a masked global load (0.0f where the mask is false), a ``dot`` (an
  ordered ``fma`` chain from 0.0f), an ``fma``, a sum of two terms, or a constant;
* threadgroup memory holds, per slot, the global address and mask of the load stored into it and
  the barrier phase that wrote it; a slot read by a ``dot`` must have been written before the last
  barrier and not in the current phase, and no slot is written twice in a phase or after a read in
  the same phase (race free, so the interleaving of the threads cannot matter);
* threads of a partial last group (ghosts) touch no memory: their global accesses carry the
  bound ``global x < active threads`` as one more mask atom; global stores go to one buffer.

The stored terms must then be, for every thread and store, the left fold ``((z + d_0) + d_1) +
... + d_{T-1}`` (``z`` = 0.0f, or the fold starts at ``d_0``) of dots of one length KT -- an
``fma`` chain over loads from 0.0f counts as a dot -- whose A addresses advance by 1 and B
addresses by one stride ``ldb`` along ``k = t*KT + j``, and the (A row, B column) pairs of the
stores must cover a rectangle exactly once, with the output address affine in row and column.
The program ids must shift that rectangle by whole rows/columns (or select a batch): one GEMM per
launch.  Finally every mask must be a rectangle bound: each atom a bound ``row < R``, ``col < C``
or ``k < Kb`` on the global GEMM coordinate it guards (its left side equals that coordinate plus
a constant), and the program-id-free part a prefix ``k < Kb`` of the K range (stores: all true).
``eas_sgemm_f32_tiled`` then performs, for every stored output, the same ``fma`` chains on the same
values (masked elements read as 0.0f) and the same additions in the same order: bit-identical
results.

Every step that does not hold makes the plan decline (``last_reason``), and the generic kernel
runs.
"""

from __future__ import annotations

import os
import struct
from dataclasses import dataclass
from typing import Any

import numpy as np

from ..ir import DType, IRModule, Inst, ValueRef

M32 = np.uint64(0xFFFFFFFF)
U32_LIMIT = 1 << 32
INF = 1 << 40


class Decline(Exception):
    pass


def _need(cond: bool, why: str) -> None:
    if not cond:
        raise Decline(why)


# ---------------------------------------------------------------------------
# values
# ---------------------------------------------------------------------------

@dataclass(frozen=True, eq=False)
class Mask:
    conc: np.ndarray                              # (NT,) bool: the program-id-free comparisons
    atoms: tuple[tuple[np.ndarray, np.ndarray], ...] = ()   # (lhs (4,NT), rhs (4,NT)): lhs < rhs


@dataclass(frozen=True, eq=False)
class FConst:
    bits: int


@dataclass(frozen=True, eq=False)
class FLoad:
    buf: str
    lin: np.ndarray   # (4, NT) uint64
    mask: Mask


@dataclass(frozen=True, eq=False)
class Side:
    """One operand of a dot: element k of thread t is ``buf[base[:, t] + k*step]`` where
    ``conc[t, k]`` and every atom ``lhs0[:, t] + k*lstep < rhs`` hold, else 0.0f."""

    buf: str
    base: np.ndarray       # (4, NT)
    step: int
    conc: np.ndarray       # (NT, K) bool
    atoms: tuple[tuple[np.ndarray, int, int], ...]


@dataclass(frozen=True, eq=False)
class FDot:
    a: Side
    b: Side
    k: int


@dataclass(frozen=True, eq=False)
class FFma:
    x: Any
    y: Any
    z: Any


@dataclass(frozen=True, eq=False)
class FAdd:
    x: Any
    y: Any


class _Smem:
    def __init__(self, n: int):
        self.buf = np.full(n, -1, np.int64)           # global buffer code, -1 = never written
        self.lin = np.zeros((4, n), np.uint64)
        self.conc = np.zeros(n, np.bool_)
        self.rec = np.full(n, -1, np.int64)           # index of the writing load's atom record
        self.writer = np.zeros(n, np.int64)           # thread that wrote the slot
        self.wphase = np.full(n, -1, np.int64)
        self.rphase = np.full(n, -1, np.int64)


def _pfree(x: np.ndarray) -> bool:
    return not x[1:].any()


def _bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(np.float32(v))))[0]


def _affine_k(arr: np.ndarray, what: str) -> tuple[np.ndarray, int]:
    """(4, NT, K) forms -> (form at k = 0, per-k increment) when the increment is one constant."""
    k = arr.shape[2]
    base = arr[:, :, 0]
    if k == 1:
        return base, 0
    d = (arr[:, :, 1] - base) & M32
    _need(_pfree(d) and bool((d[0] == d[0][0]).all()), f"{what} not one stride for all threads")
    step = int(d[0][0])
    ks = np.uint64(step) * np.arange(k, dtype=np.uint64)
    _need(bool((arr[1:] == base[1:, :, None]).all()) and bool((arr[0] == ((base[0][:, None] + ks) & M32)).all()),
          f"{what} not affine in k")
    return base, step


def _uniform_rhs(rhs: np.ndarray, what: str) -> int:
    """rhs (4, ...) forms: program-id free and one value everywhere."""
    _need(not rhs[1:].any(), f"{what}: bound depends on program_id")
    _need(bool((rhs[0] == rhs[0].flat[0]).all()), f"{what}: bound differs between elements")
    return int(rhs[0].flat[0])


# ---------------------------------------------------------------------------
# symbolic execution of one thread group
# ---------------------------------------------------------------------------

class _Exec:
    def __init__(self, ir: IRModule, nt: int, scalars: dict[str, int], ghost_limit: int | None = None,
                 pid_base: tuple[int, int, int] = (0, 0, 0)):
        self.ir, self.nt = ir, nt
        self.pid_base = pid_base                      # program id = pid_base + P (P from 0)
        self.scalars = scalars
        self.vals: dict[int, Any] = {}
        self.smem: dict[int, _Smem] = {}
        self.codes: dict[str, int] = {}
        self.records: list[tuple[tuple[np.ndarray, np.ndarray], ...]] = []
        self.phase = 0
        self.stores: list[tuple[str, np.ndarray, Any, Mask]] = []
        self.tvec = np.arange(nt, dtype=np.uint64)
        # threads whose global x index reaches ghost_limit touch no memory: every global access is
        # guarded by that bound as one more mask atom
        self.ghost: tuple[tuple[np.ndarray, np.ndarray], ...] = ()
        if ghost_limit is not None:
            gx = np.zeros((4, nt), np.uint64)
            gx[0] = (self.tvec + np.uint64(pid_base[0] * nt)) & M32
            gx[1] = np.uint64(nt)
            self.ghost = ((gx, self.lin_const(ghost_limit)),)

    def code(self, name: str) -> int:
        return self.codes.setdefault(name, len(self.codes))

    def name_of(self, code: int) -> str:
        return next(n for n, c in self.codes.items() if c == code)

    def u(self, ref: ValueRef) -> np.ndarray:
        v = self.vals[ref.id]
        _need(isinstance(v, np.ndarray) and v.dtype == np.uint64, f"v{ref.id} is not a u32 form")
        return v

    def concrete(self, ref: ValueRef) -> np.ndarray:
        v = self.u(ref)
        _need(_pfree(v), f"v{ref.id} depends on program_id where a concrete value is needed")
        return v[0]

    def scalar_const(self, ref: ValueRef) -> int:
        c = self.concrete(ref)
        _need(bool((c == c[0]).all()), f"v{ref.id} differs between threads")
        return int(c[0])

    def mask(self, ref: ValueRef) -> Mask:
        v = self.vals[ref.id]
        _need(isinstance(v, Mask), f"v{ref.id} is not a mask")
        return v

    def plain(self, ref: ValueRef) -> np.ndarray:
        m = self.mask(ref)
        _need(not m.atoms, f"v{ref.id}: a program_id-dependent mask used as a value")
        return m.conc

    def lin_const(self, c: np.ndarray | int) -> np.ndarray:
        out = np.zeros((4, self.nt), np.uint64)
        out[0] = np.uint64(c) & M32 if np.isscalar(c) else (c.astype(np.uint64) & M32)
        return out

    def run(self) -> None:
        for inst in self.ir.insts:
            getattr(self, "op_" + inst.op, self.op_unsupported)(inst)

    def op_unsupported(self, inst: Inst) -> None:
        raise Decline(f"op {inst.op!r} not handled")

    def op_arg(self, inst: Inst) -> None:
        name = str(inst.args[0])
        kind = next(a.kind for a in self.ir.args if a.name == name)
        if kind == "buffer":
            self.vals[inst.out.id] = ("gbuf", name)
        elif inst.out.dtype == DType.U32:
            self.vals[inst.out.id] = self.lin_const(int(self.scalars[name]) % U32_LIMIT)
        else:
            raise Decline(f"scalar argument {name} of type {inst.out.dtype}")

    def op_const(self, inst: Inst) -> None:
        v, dt = inst.args[0], inst.out.dtype
        if dt == DType.U32:
            self.vals[inst.out.id] = self.lin_const(int(v) % U32_LIMIT)
        elif dt == DType.BOOL:
            self.vals[inst.out.id] = Mask(np.full(self.nt, bool(v)))
        elif dt == DType.F32:
            self.vals[inst.out.id] = FConst(_bits(float(v)))
        else:
            raise Decline(f"const of type {dt}")

    def op_alloc_tg(self, inst: Inst) -> None:
        _need(inst.out.dtype == DType.F32, "threadgroup memory of a type other than f32")
        self.smem[inst.out.id] = _Smem(int(inst.args[0]))
        self.vals[inst.out.id] = ("smem", inst.out.id)

    def op_program_id(self, inst: Inst) -> None:
        ax = int(inst.args[0])
        out = np.zeros((4, self.nt), np.uint64)
        out[0] = np.uint64(self.pid_base[ax] % U32_LIMIT)
        out[1 + ax] = 1
        self.vals[inst.out.id] = out

    def op_thread_id(self, inst: Inst) -> None:
        ax = int(inst.args[0])
        out = np.zeros((4, self.nt), np.uint64)
        if ax == 0:
            out[0] = (self.tvec + np.uint64(self.pid_base[0] * self.nt)) & M32
            out[1] = np.uint64(self.nt)
        else:
            out[0] = np.uint64(self.pid_base[ax] % U32_LIMIT)
            out[1 + ax] = 1
        self.vals[inst.out.id] = out

    def op_tid(self, inst: Inst) -> None:
        self.vals[inst.out.id] = self.lin_const((self.tvec + np.uint64(int(inst.args[0]))) & M32)

    def op_local_id(self, inst: Inst) -> None:
        self.vals[inst.out.id] = self.lin_const(self.tvec if int(inst.args[0]) == 0 else 0)

    def op_lane_id(self, inst: Inst) -> None:
        self.vals[inst.out.id] = self.lin_const(self.tvec & np.uint64(31))

    def op_sg_id(self, inst: Inst) -> None:
        self.vals[inst.out.id] = self.lin_const(self.tvec >> np.uint64(5))

    def _arith_f(self, inst: Inst) -> bool:
        a, b = inst.args
        if a.dtype != DType.F32:
            return False
        _need(inst.op == "add", f"f32 {inst.op}")
        self.vals[inst.out.id] = FAdd(self.vals[a.id], self.vals[b.id])
        return True

    def op_add(self, inst: Inst) -> None:
        if self._arith_f(inst):
            return
        a, b = inst.args
        self.vals[inst.out.id] = (self.u(a) + self.u(b)) & M32

    def op_mul(self, inst: Inst) -> None:
        if self._arith_f(inst):
            return
        a, b = self.u(inst.args[0]), self.u(inst.args[1])
        if _pfree(a):
            self.vals[inst.out.id] = (a[0][None, :] * b) & M32
        elif _pfree(b):
            self.vals[inst.out.id] = (a * b[0][None, :]) & M32
        else:
            raise Decline("product of two program_id-dependent values")

    def op_fma(self, inst: Inst) -> None:
        x, y, z = inst.args
        _need(inst.out.dtype == DType.F32, "fma of a non-f32 type")
        self.vals[inst.out.id] = FFma(self.vals[x.id], self.vals[y.id], self.vals[z.id])

    def op_floordiv(self, inst: Inst) -> None:
        _need(inst.args[0].dtype == DType.U32, "non-u32 division")
        x, y = self.concrete(inst.args[0]), self.concrete(inst.args[1])
        safe = np.where(y == 0, np.uint64(1), y)
        self.vals[inst.out.id] = self.lin_const(np.where(y == 0, M32, x // safe))

    def op_mod(self, inst: Inst) -> None:
        _need(inst.args[0].dtype == DType.U32, "non-u32 remainder")
        x, y = self.concrete(inst.args[0]), self.concrete(inst.args[1])
        safe = np.where(y == 0, np.uint64(1), y)
        self.vals[inst.out.id] = self.lin_const(np.where(y == 0, x, x % safe))

    def op_lt(self, inst: Inst) -> None:
        _need(inst.args[0].dtype == DType.U32, "non-u32 comparison")
        a, b = self.u(inst.args[0]), self.u(inst.args[1])
        if _pfree(a) and _pfree(b):
            self.vals[inst.out.id] = Mask(a[0] < b[0])
        else:
            self.vals[inst.out.id] = Mask(np.ones(self.nt, np.bool_), ((a, b),))

    def op_and(self, inst: Inst) -> None:
        x, y = self.mask(inst.args[0]), self.mask(inst.args[1])
        self.vals[inst.out.id] = Mask(x.conc & y.conc, x.atoms + y.atoms)

    def op_or(self, inst: Inst) -> None:
        self.vals[inst.out.id] = Mask(self.plain(inst.args[0]) | self.plain(inst.args[1]))

    def op_not(self, inst: Inst) -> None:
        self.vals[inst.out.id] = Mask(~self.plain(inst.args[0]))

    def op_where(self, inst: Inst) -> None:
        c, a, b = inst.args
        _need(a.dtype == DType.U32, "where on a non-u32 value")
        self.vals[inst.out.id] = np.where(self.plain(c)[None, :], self.u(a), self.u(b))

    def op_barrier(self, inst: Inst) -> None:
        self.phase += 1

    def _buffer(self, ref: ValueRef) -> tuple[str, Any]:
        v = self.vals[ref.id]
        _need(isinstance(v, tuple), f"v{ref.id} is not a buffer")
        return v

    def op_load(self, inst: Inst) -> None:
        buf, off, mask = inst.args
        kind, ident = self._buffer(buf)
        _need(kind == "gbuf", "load from threadgroup memory")
        _need(inst.out.dtype == DType.F32, "load of a non-f32 value")
        m = self.mask(mask)
        self.vals[inst.out.id] = FLoad(ident, self.u(off), Mask(m.conc, m.atoms + self.ghost))

    def op_store(self, inst: Inst) -> None:
        buf, off, val, mask = inst.args
        kind, ident = self._buffer(buf)
        v = self.vals[val.id]
        m = self.mask(mask)
        if kind == "smem":
            # a program-id-free mask selects the writing threads; the others leave their slot alone
            _need(not m.atoms and not self.ghost, "threadgroup store under a program_id-dependent mask")
            sm = self.smem[ident]
            v, extra = self._slot_load(v)
            who = np.nonzero(m.conc)[0]
            s = self.concrete(off).astype(np.int64)[who]
            _need(bool((s < len(sm.buf)).all()), "threadgroup store out of range")
            _need(len(np.unique(s)) == len(s), "two threads store to one threadgroup slot")
            _need(bool((sm.wphase[s] != self.phase).all()), "threadgroup slot written twice between barriers")
            _need(bool((sm.rphase[s] != self.phase).all()), "threadgroup slot written after a read between barriers")
            sm.buf[s] = self.code(v.buf)
            sm.lin[:, s] = v.lin[:, who]
            sm.conc[s] = v.mask.conc[who]
            self.records.append(v.mask.atoms)
            sm.rec[s] = len(self.records) - 1
            sm.writer[s] = who
            sm.wphase[s] = self.phase
            self._slot_written(sm, s, extra)
        else:
            self.stores.append((ident, self.u(off), v, Mask(m.conc, m.atoms + self.ghost)))

    def _slot_load(self, v: Any) -> tuple[FLoad, Any]:
        """What a threadgroup store may write: a global load (extensions also accept e.g. its cast)."""
        _need(isinstance(v, FLoad), "threadgroup memory holds something other than a global load")
        return v, None

    def _slot_written(self, sm: _Smem, slots: np.ndarray, extra: Any) -> None:
        """Per-slot bookkeeping of extensions after a threadgroup store."""

    def _side(self, buf: ValueRef, base: ValueRef, stride: ValueRef, k: int) -> Side:
        kind, ident = self._buffer(buf)
        step = self.scalar_const(stride)
        if kind == "gbuf":
            return Side(ident, self.u(base), step, np.ones((self.nt, k), np.bool_), ())
        sm = self.smem[ident]
        b0 = self.concrete(base).astype(np.int64)
        slots = b0[:, None] + np.arange(k, dtype=np.int64)[None, :] * step   # (NT, K), exact
        _need(bool(((slots >= 0) & (slots < len(sm.buf))).all()), "dot reads outside threadgroup memory")
        _need(bool((sm.wphase[slots] >= 0).all()), "dot reads an unwritten threadgroup slot")
        _need(bool((sm.wphase[slots] < self.phase).all()), "dot reads a slot written since the last barrier")
        codes = sm.buf[slots]
        _need(bool((codes == codes.flat[0]).all()), "dot reads slots loaded from different buffers")
        sm.rphase[slots.ravel()] = self.phase
        lin_base, lstep = _affine_k(sm.lin[:, slots], "dot addresses")
        rec, writer = sm.rec[slots], sm.writer[slots]
        recs = np.unique(rec)
        na = len(self.records[int(recs[0])])
        _need(all(len(self.records[int(r)]) == na for r in recs), "slots loaded under different mask shapes")
        atoms = []
        for a in range(na):
            lhs = np.zeros((4,) + slots.shape, np.uint64)
            rhs = np.zeros((4,) + slots.shape, np.uint64)
            for r in recs:
                pos = rec == r
                l_r, r_r = self.records[int(r)][a]
                lhs[:, pos] = l_r[:, writer[pos]]
                rhs[:, pos] = r_r[:, writer[pos]]
            l0, ls = _affine_k(lhs, "mask bound")
            atoms.append((l0, ls, _uniform_rhs(rhs, "mask")))
        return Side(self.name_of(int(codes.flat[0])), lin_base, lstep, sm.conc[slots], tuple(atoms))

    def op_dot(self, inst: Inst) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, k_ref = inst.args
        _need(a_buf.dtype == DType.F32 and b_buf.dtype == DType.F32, "dot over non-f32 operands")
        k = self.scalar_const(k_ref)
        _need(k >= 1, "dot of length 0")
        self.vals[inst.out.id] = FDot(self._side(a_buf, a_base, a_stride, k), self._side(b_buf, b_base, b_stride, k), k)


# ---------------------------------------------------------------------------
# GEMM derivation
# ---------------------------------------------------------------------------

def _loads_side(loads: list[FLoad]) -> Side:
    """Global loads l_0 .. l_{K-1} (one per k) as one dot operand."""
    _need(all(isinstance(x, FLoad) for x in loads), "fma operand is not a global load")
    _need(len({x.buf for x in loads}) == 1, "fma operands from different buffers along k")
    base, step = _affine_k(np.stack([x.lin for x in loads], axis=2), "fma operand addresses")
    na = len(loads[0].mask.atoms)
    _need(all(len(x.mask.atoms) == na for x in loads), "fma operands under different mask shapes")
    atoms = []
    for a in range(na):
        l0, ls = _affine_k(np.stack([x.mask.atoms[a][0] for x in loads], axis=2), "mask bound")
        atoms.append((l0, ls, _uniform_rhs(np.stack([x.mask.atoms[a][1] for x in loads], axis=2), "mask")))
    conc = np.stack([x.mask.conc for x in loads], axis=1)
    return Side(loads[0].buf, base, step, conc, tuple(atoms))


def _as_dot(term: Any) -> FDot | None:
    """A dot, or an fma chain fma(x_{K-1}, y_{K-1}, ... fma(x_0, y_0, 0.0f)) over global loads."""
    if isinstance(term, FDot):
        return term
    if not isinstance(term, FFma):
        return None
    xs, ys = [], []
    while isinstance(term, FFma):
        xs.append(term.x)
        ys.append(term.y)
        term = term.z
    _need(isinstance(term, FConst) and term.bits == 0, "fma chain does not start at +0.0f")
    return FDot(_loads_side(xs[::-1]), _loads_side(ys[::-1]), len(xs))


def _fold(term: Any) -> tuple[bool, list[FDot]]:
    """((z + d0) + d1) + ...  ->  (zero_init, [d0, d1, ...]); IEEE addition commutes exactly."""
    chain: list[FDot] = []
    while isinstance(term, FAdd):
        dx, dy = _as_dot(term.x), _as_dot(term.y)
        if dy is not None:
            chain.append(dy)
            term = term.x
        elif dx is not None:
            chain.append(dx)
            term = term.y
        else:
            raise Decline("sum of two non-dot terms")
    d = _as_dot(term)
    if d is not None:
        chain.append(d)
        return False, chain[::-1]
    _need(isinstance(term, FConst) and term.bits == 0, "sum does not start at +0.0f or a dot")
    _need(bool(chain), "store of a constant")
    return True, chain[::-1]


def _ap(values: np.ndarray) -> tuple[int, int, int] | None:
    """Sorted distinct values as first + i*step: (first, step, count)."""
    u = np.unique(values)
    if len(u) == 1:
        return int(u[0]), 0, 1
    d = np.diff(u)
    if not (d == d[0]).all():
        return None
    return int(u[0]), int(d[0]), len(u)


def derive(ex: _Exec) -> dict[str, Any]:
    _need(bool(ex.stores), "no global stores")
    outs = {s[0] for s in ex.stores}
    _need(len(outs) == 1, "stores to more than one buffer")
    c_buf = outs.pop()
    folds = [_fold(v) for _, _, v, _ in ex.stores]
    zero_init = folds[0][0]
    _need(all(z == zero_init for z, _ in folds), "sums start differently")
    ntile = len(folds[0][1])
    _need(all(len(ch) == ntile for _, ch in folds), "sums of different lengths")
    # operand roles: A is the side contiguous along k (products commute exactly)
    d0 = folds[0][1][0]
    swap = d0.a.step != 1 and d0.b.step == 1
    chains = [[FDot(d.b, d.a, d.k) if swap else d for d in ch] for _, ch in folds]
    kt = chains[0][0].k
    _need(kt % 8 == 0, "K tile not a multiple of 8")
    a_buf, b_buf = chains[0][0].a.buf, chains[0][0].b.buf
    _need(c_buf not in (a_buf, b_buf), "output buffer is also an operand")
    base_a = np.stack([ch[0].a.base for ch in chains])          # (S, 4, NT)
    base_b = np.stack([ch[0].b.base for ch in chains])
    out_c = np.stack([s[1] for s in ex.stores])
    b_sk = chains[0][0].b.step
    for s, ch in enumerate(chains):
        for t, d in enumerate(ch):
            _need(d.k == kt and d.a.buf == a_buf and d.b.buf == b_buf, "dots differ in length or operands")
            _need(d.a.step == 1, "A not contiguous along k")
            _need(d.b.step == b_sk, "B stride along k differs")
            sh = np.uint64(t) * np.uint64(kt)
            _need(bool((((base_a[s] + np.array([sh, 0, 0, 0], np.uint64)[:, None]) & M32) == d.a.base).all()),
                  "A tiles not consecutive along k")
            _need(bool((((base_b[s] + np.array([sh * np.uint64(b_sk), 0, 0, 0], np.uint64)[:, None]) & M32)
                        == d.b.base).all()), "B tiles not consecutive along k")
    coefs = {}
    for name, arr in (("a", base_a), ("b", base_b), ("c", out_c)):
        p = arr[:, 1:, :]
        _need(bool((p == p[:1, :, :1]).all()), f"{name} address depends on program_id differently per thread")
        coefs[name] = [int(x) for x in p[0, :, 0]]
    S, NT = base_a.shape[0], base_a.shape[2]
    ca = base_a[:, 0, :].astype(np.int64)                       # (S, NT)
    cb = base_b[:, 0, :].astype(np.int64)
    cc = out_c[:, 0, :].astype(np.int64)
    ra, rb = _ap(ca.ravel()), _ap(cb.ravel())
    _need(ra is not None and rb is not None, "rows or columns not evenly spaced")
    a0, a_sm, bm = ra
    b0, b_sn, bn = rb
    _need(b_sn in (0, 1), "B columns not contiguous")
    i = (ca - a0) // a_sm if a_sm else np.zeros_like(ca)
    j = (cb - b0) // b_sn if b_sn else np.zeros_like(cb)
    _need(S * NT == bm * bn and len(np.unique((i * bn + j).ravel())) == bm * bn, "outputs do not cover the tile once")
    c0 = int(cc[(i == 0) & (j == 0)][0])
    c_sn = int(cc[(i == 0) & (j == 1)][0]) - c0 if bn > 1 else 1
    c_sm = int(cc[(i == 1) & (j == 0)][0]) - c0 if bm > 1 else 0
    _need(c_sn == 1, "C columns not contiguous")
    _need(bool((cc == c0 + i * c_sm + j * c_sn).all()), "output addresses not affine in row and column")
    return {"a_buf": a_buf, "b_buf": b_buf, "c_buf": c_buf, "zero_init": zero_init, "kt": kt, "ntile": ntile,
            "a0": a0, "a_sm": a_sm, "b0": b0, "b_sk": b_sk, "c0": c0, "c_sm": c_sm, "bm": bm, "bn": bn,
            "coef_a": coefs["a"], "coef_b": coefs["b"], "coef_c": coefs["c"],
            "_chains": chains, "_i": i, "_j": j, "_store_masks": [s[3] for s in ex.stores]}


def map_grid(d: dict[str, Any], programs: tuple[int, int, int]) -> dict[str, Any]:
    """Turn the per-group rectangle and the program-id shifts into one (batched) GEMM."""
    bm, bn = d["bm"], d["bn"]
    M, N, batch = bm, bn, 1
    row = col = bat = None
    a_sm, c_sm = d["a_sm"], d["c_sm"]
    for ax in range(3):
        if programs[ax] <= 1:
            continue
        ca, cb, cc = d["coef_a"][ax], d["coef_b"][ax], d["coef_c"][ax]
        if row is None and cb == 0 and ca != 0 and (
                (bm > 1 and ca == bm * a_sm and cc == bm * c_sm) or (bm == 1 and (a_sm, c_sm) == (0, 0))):
            row = ax
            if bm == 1:  # one row per group: the row strides are the program-id coefficients
                a_sm, c_sm = ca, cc
        elif col is None and ca == 0 and cb == bn and cc == bn:
            col = ax
        elif bat is None:
            bat = ax
        else:
            raise Decline("program ids do not map onto rows, columns and one batch axis")
    if row is not None:
        M = bm * programs[row]
    if col is not None:
        N = bn * programs[col]
    a_bs = b_bs = c_bs = 0
    if bat is not None:
        batch = programs[bat]
        a_bs, b_bs, c_bs = d["coef_a"][bat], d["coef_b"][bat], d["coef_c"][bat]
    return {"M": M, "N": N, "K": d["kt"] * d["ntile"], "batch": batch, "a_sm": a_sm, "c_sm": c_sm,
            "a_bs": a_bs, "b_bs": b_bs, "c_bs": c_bs, "row_ax": row, "col_ax": col, "bat_ax": bat}


def _classify(lhs0: np.ndarray, lstep: int, rhs: int, coords: dict[str, tuple[np.ndarray, int, int, int]],
              active: list[int], allowed: tuple[str, ...], what: str) -> tuple[str, int]:
    """An atom ``lhs0 + k*lstep < rhs`` over elements (forms broadcast to the coordinate arrays) as
    ``coord < bound``: its left side must be coordinate + a constant, with the coordinate's
    program-id coefficient and no other, and coordinate + constant must stay below 2^32 over the
    whole launch (so the u32 comparison is the integer one).  coords: name -> (per-element offset,
    program axis or -1, coefficient per program id, largest value of the coordinate in the launch),
    the coordinate's value being offset + coefficient * P[axis]."""
    for name in allowed:
        off, ax, coef, top = coords[name]
        kstep = 1 if name == "k" else 0
        if lstep != kstep:
            continue
        ok = True
        for a in active:
            want = coef if a == ax else 0
            if not bool((lhs0[1 + a] == np.uint64(want % U32_LIMIT)).all()):
                ok = False
                break
        if not ok:
            continue
        delta = (lhs0[0].astype(np.int64) - np.broadcast_to(off, lhs0[0].shape)) % U32_LIMIT
        if not bool((delta == delta.flat[0]).all()):
            continue
        dlt = int(delta.flat[0])
        if top + dlt >= U32_LIMIT:
            continue
        return name, max(0, rhs - dlt)
    raise Decline(f"{what}: a mask that is not a row, column or k bound")


def bounds(d: dict[str, Any], programs: tuple[int, int, int]) -> dict[str, int]:
    """Zero-fill and store bounds of the launch from the masks (module docstring)."""
    active = [ax for ax in range(3) if programs[ax] > 1]
    kt, bm, bn = d["kt"], d["bm"], d["bn"]
    row_ax = d["row_ax"] if d["row_ax"] is not None else -1
    col_ax = d["col_ax"] if d["col_ax"] is not None else -1
    out = {"a_rows": INF, "a_cols": INF, "a_k": INF, "b_rows": INF, "b_cols": INF, "b_k": INF, "s_rows": INF,
           "s_cols": INF}
    i, j = d["_i"], d["_j"]                                      # (S, NT)
    top_row = int(i.max()) + (bm * (programs[row_ax] - 1) if row_ax >= 0 else 0)
    top_col = int(j.max()) + (bn * (programs[col_ax] - 1) if col_ax >= 0 else 0)
    top_k = kt * d["ntile"] - 1
    for s, ch in enumerate(d["_chains"]):
        for t, dot in enumerate(ch):
            kglob = t * kt + np.arange(kt, dtype=np.int64)[None, :]   # (1, K)
            coords = {"row": (i[s][:, None], row_ax, bm, top_row), "col": (j[s][:, None], col_ax, bn, top_col),
                      "k": (kglob, -1, 0, top_k)}
            for side, pre, lim_k in ((dot.a, "a_", "a_k"), (dot.b, "b_", "b_k")):
                for l0, ls, rhs in side.atoms:
                    lhs = l0[:, :, None] + np.zeros((1, 1, kt), np.uint64)
                    kind, bound = _classify(lhs, ls, rhs, coords, active, ("row", "col", "k"), "operand mask")
                    key = lim_k if kind == "k" else pre + ("rows" if kind == "row" else "cols")
                    out[key] = min(out[key], bound)
                # the program-id-free part must be a prefix of the K range
                conc = side.conc
                kk = np.broadcast_to(kglob, conc.shape)
                if not bool(conc.all()):
                    first_false = int(kk[~conc].min())
                    _need(bool((conc == (kk < first_false)).all()), "operand mask is not a K prefix")
                    out[lim_k] = min(out[lim_k], first_false)
    for s, m in enumerate(d["_store_masks"]):
        _need(bool(m.conc.all()), "store mask with a program_id-free part")
        coords = {"row": (i[s], row_ax, bm, top_row), "col": (j[s], col_ax, bn, top_col)}
        for lhs, rhs in m.atoms:
            kind, bound = _classify(lhs, 0, _uniform_rhs(rhs, "store mask"), coords, active, ("row", "col"),
                                    "store mask")
            key = "s_rows" if kind == "row" else "s_cols"
            out[key] = min(out[key], bound)
    return out


def plan_launch(d: dict[str, Any], g: dict[str, Any], b: dict[str, int]) -> dict[str, Any]:
    """Extents, zero-fill bounds and address limits of the native launch."""
    M = min(g["M"], b["s_rows"])
    N = min(g["N"], b["s_cols"])
    K, batch = g["K"], g["batch"]
    # a bound on A by the output column (or on B by the output row) only holds if no stored output
    # lies beyond it: then it is true wherever the result is kept
    _need(b["a_cols"] >= N and b["b_rows"] >= M, "operand masked by the other operand's coordinate")
    a_rows, b_cols = min(M, b["a_rows"]), min(N, b["b_cols"])
    a_k, b_k = min(K, b["a_k"]), min(K, b["b_k"])
    a_sm, c_sm = g["a_sm"], g["c_sm"]
    _need(M <= 1 or c_sm >= N, "output rows overlap")
    _need(batch == 1 or g["c_bs"] >= (M - 1) * c_sm + N, "output batches overlap")
    top_a = d["a0"] + max(a_rows - 1, 0) * a_sm + max(a_k - 1, 0) + (batch - 1) * g["a_bs"]
    top_b = d["b0"] + max(b_k - 1, 0) * d["b_sk"] + max(b_cols - 1, 0) + (batch - 1) * g["b_bs"]
    top_c = d["c0"] + max(M - 1, 0) * c_sm + max(N - 1, 0) + (batch - 1) * g["c_bs"]
    _need(max(top_a, top_b, top_c) < U32_LIMIT, "an index would wrap at 2^32")
    out = {k: v for k, v in d.items() if not k.startswith("_")}
    out.update({"M": M, "N": N, "K": K, "batch": batch, "a_sm": a_sm, "c_sm": c_sm, "a_bs": g["a_bs"],
                "b_bs": g["b_bs"], "c_bs": g["c_bs"], "a_rows": a_rows, "a_k": a_k, "b_cols": b_cols, "b_k": b_k,
                "top_a": top_a, "top_b": top_b, "top_c": top_c,
                "empty": M <= 0 or N <= 0,
                "reads_a": a_rows > 0 and a_k > 0, "reads_b": b_cols > 0 and b_k > 0})
    return out


# ---------------------------------------------------------------------------
# plan
# ---------------------------------------------------------------------------

_OPS = {"arg", "const", "alloc_tg", "program_id", "thread_id", "tid", "local_id", "lane_id", "sg_id", "add", "mul",
        "floordiv", "mod", "lt", "and", "or", "not", "where", "barrier", "load", "store", "dot", "fma"}


_SRC_HASHES: dict[str, str] = {}


def _src_hash(path: str) -> str:
    import hashlib

    if path not in _SRC_HASHES:
        _SRC_HASHES[path] = hashlib.sha256(open(path, "rb").read()).hexdigest()
    return _SRC_HASHES[path]


class ProvenGemmPlan:
    """Per-launch proof (a symbolic execution, cached in memory and on disk) and the checks every
    native GEMM launch shares; subclasses give the executor and the launch itself."""

    kind = ""
    executor: type = _Exec
    allow_ghosts = True

    def __init__(self, ir: IRModule, block: int):
        self.ir = ir
        self.block = block
        self.cache: dict[Any, Any] = {}
        self.last_reason = ""

    def _disk_path(self, key: tuple) -> Any:
        """Cache file of one proof result under EAS_CACHE_DIR/plans (None when caching is off).  The
        key hashes the IR, the launch values and the proof's own source files, so a change of the
        proof logic never reuses an old result."""
        import hashlib
        import json
        import sys

        from ..ir import ir_to_json
        from ..runtime.cuda import _cache_dir

        cdir = _cache_dir()
        if cdir is None or os.environ.get("EAS_PLAN_CACHE", "1") == "0":
            return None
        h = hashlib.sha256()
        for mod in {__name__, type(self).__module__}:
            h.update(_src_hash(sys.modules[mod].__file__).encode())
        h.update(json.dumps([self.kind, ir_to_json(self.ir), self.block, repr(key)], separators=(",", ":")).encode())
        return cdir / "plans" / f"{h.hexdigest()}.json"

    def analyse(self, scalars: dict[str, int], programs: tuple[int, int, int], ntx: int,
                pid_base: tuple[int, int, int] = (0, 0, 0)) -> dict[str, Any] | None:
        """Proof and launch values for the programs ``pid_base + [0, programs)``."""
        import json

        key = (tuple(sorted(scalars.items())), programs, ntx, tuple(pid_base))
        hit = self.cache.get(key)
        disk = None
        if hit is None:
            disk = self._disk_path(key)
            if disk is not None and disk.exists():
                try:
                    hit = json.loads(disk.read_text())["result"]
                except (OSError, ValueError, KeyError):
                    hit = None
        if hit is None:
            try:
                ghost = ntx if ntx < (pid_base[0] + programs[0]) * self.block else None
                _need(ghost is None or self.allow_ghosts, "partial thread groups")
                ex = self.executor(self.ir, self.block, scalars, ghost, tuple(pid_base))
                ex.run()
                d = derive(ex)
                g = map_grid(d, programs)
                d.update({"row_ax": g["row_ax"], "col_ax": g["col_ax"]})
                hit = plan_launch(d, g, bounds(d, programs))
            except Decline as e:
                hit = str(e)
            if disk is not None:
                try:
                    disk.parent.mkdir(parents=True, exist_ok=True)
                    tmp = disk.with_suffix(f".{os.getpid()}.tmp")
                    tmp.write_text(json.dumps({"result": hit}))
                    os.replace(tmp, disk)
                except OSError:
                    pass
        if len(self.cache) > 64:
            self.cache.clear()
        self.cache[key] = hit
        if isinstance(hit, str):
            self.last_reason = hit
            return None
        return hit

    def try_launch(self, rt: Any, ck: Any, runtime_args: dict[str, Any], args: dict[str, Any], device: int,
                   stream: int, programs: tuple[int, int, int], ntx: int, pid_base: tuple[int, int, int] = (0, 0, 0),
                   elem_base: dict[str, int] | None = None) -> bool:
        """Launch for programs ``pid_base + [0, programs)``; buffers in ``elem_base`` hold only the
        elements from that global index on (pointers already moved back by it).  False (and
        ``last_reason``) when the proof or a check fails: the caller runs the generated kernel."""
        if os.environ.get("EAS_DISABLE_NATIVE", "0") not in ("", "0"):
            self.last_reason = "disabled by EAS_DISABLE_NATIVE"
            return False
        scalars = {a.name: int(runtime_args[a.name]) for a in self.ir.args
                   if a.kind == "scalar" and a.dtype == DType.U32}
        d = self.analyse(scalars, programs, ntx, pid_base)
        if d is None:
            return False
        if d["empty"]:
            return True  # the kernel stores nothing for these values
        from .patterns import _numel

        eb = elem_base or {}
        for n, lo, top, used in ((d["a_buf"], d["a0"], d["top_a"], d["reads_a"]),
                                 (d["b_buf"], d["b0"], d["top_b"], d["reads_b"]), (d["c_buf"], d["c0"], d["top_c"], True)):
            e = int(eb.get(n, 0))
            if used and (lo < e or top >= e + _numel(runtime_args[n])):
                self.last_reason = f"{n}: the product reaches outside the buffer"
                return False
        pa, pb, pc = args[d["a_buf"]].ptr, args[d["b_buf"]].ptr, args[d["c_buf"]].ptr
        c_lo, c_hi = pc + 4 * d["c0"], pc + 4 * (d["top_c"] + 1)
        for p, top in ((pa, d["top_a"]), (pb, d["top_b"])):
            if p < c_hi and c_lo < p + 4 * (top + 1):
                self.last_reason = "output overlaps an operand"
                return False
        return self._launch(rt, d, pa, pb, pc, device, stream)

    def _launch(self, rt: Any, d: dict[str, Any], pa: int, pb: int, pc: int, device: int, stream: int) -> bool:
        raise NotImplementedError

    def covers(self, runtime_args: dict[str, Any], programs: tuple[int, int, int], ntx: int, name: str,
               numel: int) -> bool:
        """True when this launch stores every element of buffer ``name`` (numel elements from index 0):
        the proven output rectangle M x N of every batch is one dense block starting at 0."""
        scalars = {a.name: int(runtime_args[a.name]) for a in self.ir.args
                   if a.kind == "scalar" and a.dtype == DType.U32}
        d = self.analyse(scalars, programs, ntx)
        if d is None or d["empty"] or d["c_buf"] != name:
            return False
        M, N, B = d["M"], d["N"], d["batch"]
        dense = (M == 1 or d["c_sm"] == N) and (B == 1 or d["c_bs"] == M * N)
        return dense and d["c0"] == 0 and M * N * B == numel


class TiledGemmPlan(ProvenGemmPlan):
    """Native FFMA launch for kernels proven to be tiled fp32 GEMMs (module docstring)."""

    kind = "tiled_f32_ffma"
    last_mode = ""

    def _launch(self, rt: Any, d: dict[str, Any], pa: int, pb: int, pc: int, device: int, stream: int) -> bool:
        from ..runtime import cuda_ext

        if fp32_mode() == "3xtf32" and self._launch_3xtf32(rt, d, pa, pb, pc, device, stream):
            return True
        rc = rt.lib().eas_sgemm_f32_tiled(pa + 4 * d["a0"], pb + 4 * d["b0"], pc + 4 * d["c0"], d["M"], d["N"], d["K"],
                                          d["kt"], d["batch"], d["a_sm"], d["a_bs"], d["b_sk"], d["b_bs"], d["c_sm"],
                                          d["c_bs"], int(d["zero_init"]), d["a_rows"], d["a_k"], d["b_cols"],
                                          d["b_k"], stream)
        if rc == cuda_ext.EAS_ERR_VALUE:
            self.last_reason = cuda_ext.last_error()
            return False
        cuda_ext.check(rc, "sgemm_f32_tiled (FFMA)")
        rt.launch_count += 1
        rt.native_launches += 1
        self.last_mode = "exact"
        return True


    def _launch_3xtf32(self, rt: Any, d: dict[str, Any], pa: int, pb: int, pc: int, device: int,
                       stream: int) -> bool:
        """Opt-in 3xTF32 mode: C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi as ONE tcgen05 kind::tf32 GEMM.
        eas_split_tf32 writes each row of A and each column of B (K-major) as [hi | lo] segments of
        kp = K rounded up to 32 (zero outside the proof's bounds); the GEMM's producer maps its
        3 kp/32 k-blocks onto the segment pairs (hi, hi), (hi, lo), (lo, hi).  Not bit-identical to
        the kernel's own fma chains: the dropped A_lo.B_lo term is 2^-22 of a product and the tensor
        core rounds its accumulator once per 8-deep MMA, so the error grows with K (~3e-5 normwise
        at K = 2048), inside the fp32 matmul tolerance rtol 1e-4.  False (FFMA runs instead) when
        the operands cannot be staged or the GEMM declines the shape."""
        from ..runtime import cuda_ext

        M, N, K, batch = d["M"], d["N"], d["K"], d["batch"]
        kp = -(-K // 32) * 32
        sa = rt.scratch(device, stream, "tf32_a2", 4 * batch * M * 2 * kp)
        sb = rt.scratch(device, stream, "tf32_b2", 4 * batch * N * 2 * kp)
        if sa is None or sb is None or K == 0:
            return False
        (a2, _keep_a), (b2, _keep_b) = sa, sb
        lib = rt.lib()
        cuda_ext.check(lib.eas_split_tf32(pa + 4 * d["a0"], a2, M, kp, d["a_sm"], d["a_rows"], d["a_k"], batch,
                                          d["a_bs"], 0, stream), "split A into tf32 pairs")
        cuda_ext.check(lib.eas_split_tf32(pb + 4 * d["b0"], b2, N, kp, d["b_sk"], d["b_cols"], d["b_k"], batch,
                                          d["b_bs"], 1, stream), "split B into tf32 pairs")
        rc = lib.eas_gemm_3xtf32(a2, b2, pc + 4 * d["c0"], M, N, kp, batch, 2 * kp, 2 * M * kp, 2 * kp, 2 * N * kp,
                                 d["c_sm"] if M > 1 else N, d["c_bs"], 256 if M > 128 else 128, stream)
        if rc == cuda_ext.EAS_ERR_VALUE:
            self.last_reason = cuda_ext.last_error()
            return False
        cuda_ext.check(rc, "gemm_3xtf32 (tcgen05)")
        rt.launch_count += 3
        rt.native_launches += 1
        self.last_mode = "3xtf32"
        return True


def fp32_mode() -> str:
    """EAS_FP32_MATMUL: "exact" (default; the FFMA kernel repeats the kernel's fma chains bit for
    bit) or "3xtf32" (tensor cores, within rtol 1e-4 of the exact product)."""
    m = os.environ.get("EAS_FP32_MATMUL", "exact").strip().lower() or "exact"
    if m not in ("exact", "3xtf32"):
        raise ValueError(f"EAS_FP32_MATMUL must be 'exact' or '3xtf32', not {m!r}")
    return m


def match_tiled(ir: IRModule, lowered: Any) -> TiledGemmPlan | None:
    """Cheap static filter; the proof runs per launch."""
    if lowered.mode != "thread":
        return None
    if any(i.op not in _OPS for i in ir.insts):
        return None
    if not any(i.op in ("dot", "fma") for i in ir.insts):
        return None
    if any(i.op == "fma" and i.out.dtype != DType.F32 for i in ir.insts):
        return None
    return TiledGemmPlan(ir, lowered.block_size)
