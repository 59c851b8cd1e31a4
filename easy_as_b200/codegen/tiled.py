"""Prove that a thread-mode kernel is a tiled fp32 GEMM, and launch the native FFMA kernel for it.

Target: the reference's fp32 tiled matmul (easy_as
``examples/matmul_tiled.py:134-230``): threads copy A and B tiles into
threadgroup memory, a barrier, then each thread runs ``mk.dot`` over the tiles
for its outputs and adds the dot to a running sum, tile after tile; finally it
stores the sums.  The generic lowering reproduces that thread structure, so it
is bound by shared-memory reads (one row by four columns per thread).

Nothing here matches source text or instruction order.  For a given launch
(scalar argument values, grid, threads per group) the whole thread group is
executed symbolically, all threads at once:

* every u32 value is, per thread, a linear form ``c + a0*P0 + a1*P1 + a2*P2``
  modulo 2^32 in the program ids (numpy arrays over the threads); products,
  divisions, remainders and comparisons need at least one operand free of the
  program ids, so the forms stay linear and the divisions exact;
* a float value is a term: a global load at a linear address, a ``dot`` (an
  ordered ``fma`` chain from 0.0f), a sum of two terms, or a constant;
* threadgroup memory holds, per slot, the global address its value was
  loaded from and the barrier phase that wrote it; a slot read by a ``dot`` must
  have been written before the last barrier and not in the current phase, and
  no slot is written twice in a phase or after a read in the same phase (race
  free, so the threads' interleaving cannot matter);
* masks must be true for every thread, there are no ghost threads, and the only
  global stores are the final sums.

The stored terms must then be, for every thread and store, the left fold
``((z + d_0) + d_1) + ... + d_{T-1}`` (``z`` = 0.0f, or the fold starts at
``d_0``) of dots of one length KT whose A addresses advance by 1 and B
addresses by a constant ``ldb`` along ``k = t*KT + j``, and the (A row, B
column) pairs of the threads' stores must cover a rectangle exactly once, with
the output address affine in the row and column indices.  The program ids
shift that rectangle by whole rows/columns (or select a batch), which gives one
GEMM for the whole launch.  ``eas_sgemm_f32_tiled`` then performs, for every
output, the same ``fma`` chains and additions in the same order: bit-identical
results.

Every step that does not hold makes the plan decline (``last_reason``), and
the generic kernel runs.
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


class Decline(Exception):
    pass


def _need(cond: bool, why: str) -> None:
    if not cond:
        raise Decline(why)


# ---------------------------------------------------------------------------
# float terms
# ---------------------------------------------------------------------------

@dataclass(frozen=True, eq=False)
class FConst:
    bits: int


@dataclass(frozen=True, eq=False)
class FLoad:
    buf: str
    lin: np.ndarray  # (4, NT) uint64


@dataclass(frozen=True, eq=False)
class FDot:
    a_buf: str
    a_base: np.ndarray   # (4, NT) global element address of k = 0
    a_step: int          # address increment per k (same for all threads)
    b_buf: str
    b_base: np.ndarray
    b_step: int
    k: int


@dataclass(frozen=True, eq=False)
class FAdd:
    x: Any
    y: Any


class _Smem:
    def __init__(self, n: int):
        self.buf = np.full(n, -1, np.int64)           # global buffer code, -1 = never written
        self.lin = np.zeros((4, n), np.uint64)
        self.wphase = np.full(n, -1, np.int64)
        self.rphase = np.full(n, -1, np.int64)


def _pfree(x: np.ndarray) -> bool:
    return not x[1:].any()


def _bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(np.float32(v))))[0]


# ---------------------------------------------------------------------------
# symbolic execution of one thread group
# ---------------------------------------------------------------------------

class _Exec:
    def __init__(self, ir: IRModule, nt: int, scalars: dict[str, int]):
        self.ir, self.nt = ir, nt
        self.scalars = scalars
        self.vals: dict[int, Any] = {}
        self.smem: dict[int, _Smem] = {}
        self.gbuf: dict[int, str] = {}
        self.codes: dict[str, int] = {}
        self.phase = 0
        self.stores: list[tuple[str, np.ndarray, Any]] = []
        self.tvec = np.arange(nt, dtype=np.uint64)

    def code(self, name: str) -> int:
        return self.codes.setdefault(name, len(self.codes))

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

    def mask_true(self, ref: ValueRef) -> None:
        v = self.vals[ref.id]
        _need(isinstance(v, np.ndarray) and v.dtype == np.bool_ and bool(v.all()), "mask not true for every thread")

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
            self.gbuf[inst.out.id] = name
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
            self.vals[inst.out.id] = np.full(self.nt, bool(v))
        elif dt == DType.F32:
            self.vals[inst.out.id] = FConst(_bits(float(v)))
        else:
            raise Decline(f"const of type {dt}")

    def op_alloc_tg(self, inst: Inst) -> None:
        _need(inst.out.dtype == DType.F32, "threadgroup memory of a type other than f32")
        self.smem[inst.out.id] = _Smem(int(inst.args[0]))
        self.vals[inst.out.id] = ("smem", inst.out.id)

    def op_program_id(self, inst: Inst) -> None:
        out = np.zeros((4, self.nt), np.uint64)
        out[1 + int(inst.args[0])] = 1
        self.vals[inst.out.id] = out

    def op_thread_id(self, inst: Inst) -> None:
        ax = int(inst.args[0])
        out = np.zeros((4, self.nt), np.uint64)
        if ax == 0:
            out[0] = self.tvec
            out[1] = np.uint64(self.nt)
        else:
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
        self.vals[inst.out.id] = self.concrete(inst.args[0]) < self.concrete(inst.args[1])

    def _bool(self, ref: ValueRef) -> np.ndarray:
        v = self.vals[ref.id]
        _need(isinstance(v, np.ndarray) and v.dtype == np.bool_, f"v{ref.id} is not a mask")
        return v

    def op_and(self, inst: Inst) -> None:
        self.vals[inst.out.id] = self._bool(inst.args[0]) & self._bool(inst.args[1])

    def op_or(self, inst: Inst) -> None:
        self.vals[inst.out.id] = self._bool(inst.args[0]) | self._bool(inst.args[1])

    def op_not(self, inst: Inst) -> None:
        self.vals[inst.out.id] = ~self._bool(inst.args[0])

    def op_where(self, inst: Inst) -> None:
        c, a, b = inst.args
        _need(a.dtype == DType.U32, "where on a non-u32 value")
        cond = self._bool(c)
        self.vals[inst.out.id] = np.where(cond[None, :], self.u(a), self.u(b))

    def op_barrier(self, inst: Inst) -> None:
        self.phase += 1

    def _buffer(self, ref: ValueRef) -> tuple[str, Any]:
        v = self.vals[ref.id]
        _need(isinstance(v, tuple), f"v{ref.id} is not a buffer")
        return v

    def op_load(self, inst: Inst) -> None:
        buf, off, mask = inst.args
        self.mask_true(mask)
        kind, ident = self._buffer(buf)
        _need(kind == "gbuf", "load from threadgroup memory")
        _need(inst.out.dtype == DType.F32, "load of a non-f32 value")
        self.vals[inst.out.id] = FLoad(ident, self.u(off))

    def op_store(self, inst: Inst) -> None:
        buf, off, val, mask = inst.args
        self.mask_true(mask)
        kind, ident = self._buffer(buf)
        v = self.vals[val.id]
        if kind == "smem":
            sm = self.smem[ident]
            _need(isinstance(v, FLoad), "threadgroup memory holds something other than a global load")
            slots = self.concrete(off)
            _need(bool((slots < len(sm.buf)).all()), "threadgroup store out of range")
            s = slots.astype(np.int64)
            _need(len(np.unique(s)) == len(s), "two threads store to one threadgroup slot")
            _need(bool((sm.wphase[s] != self.phase).all()), "threadgroup slot written twice between barriers")
            _need(bool((sm.rphase[s] != self.phase).all()), "threadgroup slot written after a read between barriers")
            sm.buf[s] = self.code(v.buf)
            sm.lin[:, s] = v.lin
            sm.wphase[s] = self.phase
        else:
            self.stores.append((ident, self.u(off), v))

    def _dot_side(self, buf: ValueRef, base: ValueRef, stride: ValueRef, k: int) -> tuple[str, np.ndarray, int]:
        kind, ident = self._buffer(buf)
        step = self.scalar_const(stride)
        if kind == "gbuf":
            return ident, self.u(base), step
        sm = self.smem[ident]
        b0 = self.concrete(base).astype(np.int64)
        slots = b0[:, None] + np.arange(k, dtype=np.int64)[None, :] * step   # (NT, K), exact
        _need(bool(((slots >= 0) & (slots < len(sm.buf))).all()), "dot reads outside threadgroup memory")
        _need(bool((sm.wphase[slots] >= 0).all()), "dot reads an unwritten threadgroup slot")
        _need(bool((sm.wphase[slots] < self.phase).all()), "dot reads a slot written since the last barrier")
        codes = sm.buf[slots]
        _need(bool((codes == codes.flat[0]).all()), "dot reads slots loaded from different buffers")
        sm.rphase[slots.ravel()] = self.phase
        lin = sm.lin[:, slots]                                   # (4, NT, K)
        base_lin = lin[:, :, 0]
        if k > 1:
            d = (lin[:, :, 1] - base_lin) & M32
            _need(_pfree(d) and bool((d[0] == d[0][0]).all()), "dot addresses not one stride for all threads")
            dk = int(d[0][0])
            want = np.repeat(base_lin[:, :, None], k, axis=2)
            want[0] = (want[0] + np.uint64(dk) * np.arange(k, dtype=np.uint64)[None, :]) & M32
            _need(bool((lin == want).all()), "dot addresses not affine in k")
        else:
            dk = 0
        name = next(n for n, c in self.codes.items() if c == int(codes.flat[0]))
        return name, base_lin, dk

    def op_dot(self, inst: Inst) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, k_ref = inst.args
        _need(a_buf.dtype == DType.F32 and b_buf.dtype == DType.F32, "dot over non-f32 operands")
        k = self.scalar_const(k_ref)
        _need(k >= 1, "dot of length 0")
        an, ab, ad = self._dot_side(a_buf, a_base, a_stride, k)
        bn, bb, bd = self._dot_side(b_buf, b_base, b_stride, k)
        self.vals[inst.out.id] = FDot(an, ab, ad, bn, bb, bd, k)


# ---------------------------------------------------------------------------
# GEMM derivation
# ---------------------------------------------------------------------------

def _fold(term: Any) -> tuple[bool, list[FDot]]:
    """((z + d0) + d1) + ...  ->  (zero_init, [d0, d1, ...])."""
    chain: list[FDot] = []
    while isinstance(term, FAdd):
        x, y = term.x, term.y
        if isinstance(y, FDot) and not isinstance(x, FDot) or (isinstance(x, FDot) and isinstance(y, FDot)):
            chain.append(y)
            term = x
        elif isinstance(x, FDot):
            chain.append(x)
            term = y
        else:
            raise Decline("sum of two non-dot terms")
    if isinstance(term, FDot):
        chain.append(term)
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
    outs = {b for b, _, _ in ex.stores}
    _need(len(outs) == 1, "stores to more than one buffer")
    c_buf = outs.pop()
    folds = [_fold(v) for _, _, v in ex.stores]
    zero_init = folds[0][0]
    _need(all(z == zero_init for z, _ in folds), "sums start differently")
    ntile = len(folds[0][1])
    _need(all(len(ch) == ntile for _, ch in folds), "sums of different lengths")
    kt = folds[0][1][0].k
    _need(kt % 8 == 0, "K tile not a multiple of 8")
    a_buf, b_buf = folds[0][1][0].a_buf, folds[0][1][0].b_buf
    _need(c_buf not in (a_buf, b_buf), "output buffer is also an operand")
    S = len(ex.stores)
    base_a = np.stack([ch[0].a_base for _, ch in folds])          # (S, 4, NT)
    base_b = np.stack([ch[0].b_base for _, ch in folds])
    out_c = np.stack([off for _, off, _ in ex.stores])
    for _, ch in folds:
        for t, d in enumerate(ch):
            _need(d.k == kt and d.a_buf == a_buf and d.b_buf == b_buf, "dots differ in length or operands")
            _need(d.a_step == 1 or kt == 1, "A not contiguous along k")
    b_sk = folds[0][1][0].b_step
    kk0 = np.uint64(kt)
    for s, (_, ch) in enumerate(folds):
        for t, d in enumerate(ch):
            _need(d.b_step == b_sk, "B stride along k differs")
            sh = np.uint64(t) * kk0
            _need(bool((((base_a[s] + np.array([sh, 0, 0, 0], np.uint64)[:, None]) & M32) == d.a_base).all()),
                  "A tiles not consecutive along k")
            _need(bool((((base_b[s] + np.array([sh * np.uint64(b_sk), 0, 0, 0], np.uint64)[:, None]) & M32)
                        == d.b_base).all()), "B tiles not consecutive along k")
    # program-id coefficients, common to every output
    coefs = {}
    for name, arr in (("a", base_a), ("b", base_b), ("c", out_c)):
        p = arr[:, 1:, :]
        _need(bool((p == p[:1, :, :1]).all()), f"{name} address depends on program_id differently per thread")
        coefs[name] = [int(x) for x in p[0, :, 0]]
    ca = base_a[:, 0, :].ravel().astype(np.int64)
    cb = base_b[:, 0, :].ravel().astype(np.int64)
    cc = out_c[:, 0, :].ravel().astype(np.int64)
    ra, rb = _ap(ca), _ap(cb)
    _need(ra is not None and rb is not None, "rows or columns not evenly spaced")
    a0, a_sm, bm = ra
    b0, b_sn, bn = rb
    _need(b_sn in (0, 1), "B columns not contiguous")
    i = (ca - a0) // a_sm if a_sm else np.zeros_like(ca)
    j = (cb - b0) // b_sn if b_sn else np.zeros_like(cb)
    _need(len(ca) == bm * bn and len(np.unique(i * bn + j)) == bm * bn, "outputs do not cover the tile once")
    c0 = int(cc[(i == 0) & (j == 0)][0])
    # C = c0 + i*c_sm + j*c_sn
    c_sn = int(cc[(i == 0) & (j == 1)][0]) - c0 if bn > 1 else 1
    c_sm = int(cc[(i == 1) & (j == 0)][0]) - c0 if bm > 1 else 0
    _need(c_sn == 1, "C columns not contiguous")
    _need(bool((cc == c0 + i * c_sm + j * c_sn).all()), "output addresses not affine in row and column")
    return {"a_buf": a_buf, "b_buf": b_buf, "c_buf": c_buf, "zero_init": zero_init, "kt": kt, "ntile": ntile,
            "a0": a0, "a_sm": a_sm, "b0": b0, "b_sk": b_sk, "c0": c0, "c_sm": c_sm, "bm": bm, "bn": bn,
            "coef_a": coefs["a"], "coef_b": coefs["b"], "coef_c": coefs["c"]}


def map_grid(d: dict[str, Any], programs: tuple[int, int, int]) -> dict[str, Any]:
    """Turn the per-group rectangle and the program-id shifts into one (batched) GEMM."""
    bm, bn = d["bm"], d["bn"]
    M, N, batch = bm, bn, 1
    row = col = bat = None
    for ax in range(3):
        if programs[ax] <= 1:
            continue
        ca, cb, cc = d["coef_a"][ax], d["coef_b"][ax], d["coef_c"][ax]
        if row is None and bm > 1 and cb == 0 and ca == bm * d["a_sm"] and cc == bm * d["c_sm"]:
            row = ax
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
    K = d["kt"] * d["ntile"]
    # outputs written once: rows apart by >= N, batches apart by the whole M x N block
    _need(M == 1 or d["c_sm"] >= N, "output rows overlap")
    _need(batch == 1 or c_bs >= (M - 1) * d["c_sm"] + N, "output batches overlap")
    top_a = d["a0"] + (M - 1) * d["a_sm"] + (K - 1) + (batch - 1) * a_bs
    top_b = d["b0"] + (K - 1) * d["b_sk"] + (N - 1) + (batch - 1) * b_bs
    top_c = d["c0"] + (M - 1) * d["c_sm"] + (N - 1) + (batch - 1) * c_bs
    _need(max(top_a, top_b, top_c) < U32_LIMIT, "an index would wrap at 2^32")
    return {"M": M, "N": N, "K": K, "batch": batch, "a_bs": a_bs, "b_bs": b_bs, "c_bs": c_bs,
            "top_a": top_a, "top_b": top_b, "top_c": top_c}


# ---------------------------------------------------------------------------
# plan
# ---------------------------------------------------------------------------

_OPS = {"arg", "const", "alloc_tg", "program_id", "thread_id", "tid", "local_id", "lane_id", "sg_id", "add", "mul",
        "floordiv", "mod", "lt", "and", "or", "not", "where", "barrier", "load", "store", "dot"}


class TiledGemmPlan:
    """Native FFMA launch for kernels proven to be tiled fp32 GEMMs (module docstring)."""

    kind = "tiled_f32_ffma"

    def __init__(self, ir: IRModule, block: int):
        self.ir = ir
        self.block = block
        self.cache: dict[Any, Any] = {}
        self.last_reason = ""

    def analyse(self, scalars: dict[str, int], programs: tuple[int, int, int], ntx: int) -> dict[str, Any] | None:
        key = (tuple(sorted(scalars.items())), programs, ntx)
        hit = self.cache.get(key)
        if hit is None:
            try:
                _need(ntx >= programs[0] * self.block, "partial thread groups (ghost threads)")
                ex = _Exec(self.ir, self.block, scalars)
                ex.run()
                d = derive(ex)
                d.update(map_grid(d, programs))
                hit = d
            except Decline as e:
                hit = str(e)
            if len(self.cache) > 64:
                self.cache.clear()
            self.cache[key] = hit
        if isinstance(hit, str):
            self.last_reason = hit
            return None
        return hit

    def try_launch(self, rt: Any, ck: Any, runtime_args: dict[str, Any], args: dict[str, Any], device: int,
                   stream: int, programs: tuple[int, int, int], ntx: int) -> bool:
        if os.environ.get("EAS_DISABLE_NATIVE", "0") not in ("", "0"):
            self.last_reason = "disabled by EAS_DISABLE_NATIVE"
            return False
        scalars = {a.name: int(runtime_args[a.name]) for a in self.ir.args
                   if a.kind == "scalar" and a.dtype == DType.U32}
        d = self.analyse(scalars, programs, ntx)
        if d is None:
            return False
        from .patterns import _numel

        for n, top in ((d["a_buf"], d["top_a"]), (d["b_buf"], d["top_b"]), (d["c_buf"], d["top_c"])):
            if top >= _numel(runtime_args[n]):
                self.last_reason = f"{n}: the product reaches past the buffer"
                return False
        pa, pb, pc = args[d["a_buf"]].ptr, args[d["b_buf"]].ptr, args[d["c_buf"]].ptr
        c_lo, c_hi = pc + 4 * d["c0"], pc + 4 * (d["top_c"] + 1)
        for p, top in ((pa, d["top_a"]), (pb, d["top_b"])):
            if p < c_hi and c_lo < p + 4 * (top + 1):
                self.last_reason = "output overlaps an operand"
                return False
        lib = rt.lib()
        rc = lib.eas_sgemm_f32_tiled(pa + 4 * d["a0"], pb + 4 * d["b0"], pc + 4 * d["c0"], d["M"], d["N"], d["K"],
                                     d["kt"], d["batch"], d["a_sm"], d["a_bs"], d["b_sk"], d["b_bs"], d["c_sm"],
                                     d["c_bs"], int(d["zero_init"]), stream)
        from ..runtime import cuda_ext

        if rc == cuda_ext.EAS_ERR_VALUE:
            self.last_reason = cuda_ext.last_error()
            return False
        cuda_ext.check(rc, "sgemm_f32_tiled (FFMA)")
        rt.launch_count += 1
        rt.native_launches += 1
        return True


def match_tiled(ir: IRModule, lowered: Any) -> TiledGemmPlan | None:
    """Cheap static filter; the proof runs per launch."""
    if lowered.mode != "thread":
        return None
    if any(i.op not in _OPS for i in ir.insts):
        return None
    if not any(i.op == "dot" for i in ir.insts):
        return None
    return TiledGemmPlan(ir, lowered.block_size)
