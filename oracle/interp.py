"""CPU oracle: a numpy interpreter of easy_as IR.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
arm use this module, always as the checker.  The product path
(``easy_as_b200``) never imports it.

The reference executes IR only on Apple GPUs through generated Metal
(``eas/codegen/msl.py``) and has no CPU backend (``eas/runtime/__init__.py:40-43``),
so this interpreter restates the execution semantics the Metal emitter and
runtime define:

* mode and BLOCK: ``arange`` -> SPMD, ``tid`` -> thread mode, one size
  (``msl.py:59-95``);
* launch geometry: ``metal.py:257-326`` with ``grid.py:11-130`` (SPMD launches
  one program per Metal thread; thread mode 1D without ``_grid`` dispatches
  exactly ``N`` threads, so the last threadgroup is partial);
* SPMD program: lane vectors, masked load yields 0, masked store skipped
  (``msl.py:309-342``), program_id/thread_id = program index;
* thread mode: ``tid = start + local x``, ``thread_id = global x``,
  ``lane = local x % 32``, ``sg = local x // 32`` (``msl.py:690-749,769-860``);
  threadgroup memory per group; all threads run in lockstep, which is a valid
  schedule for any race-free program, so barriers are no-ops here;
* arithmetic: u32 wraps mod 2**32; f32 ``add``/``mul`` round once; ``fma`` is a
  single-rounded f32 fused multiply-add (computed exactly below); f16 ops are
  computed in f32 and rounded to f16 once (``msl.py:885-897``);
* ``dot``: ``acc = 0; for k < K: acc = fma(float(a[..]), float(b[..]), acc)``
  in k order (``msl.py:920-952``);
* ``mma``: 8x8 tiles loaded row-major with element stride, ``D = A @ B + C``
  (Apple's summation order is unspecified, so the oracle sums in float64 and
  rounds once to f32; parity for ``mma`` is tolerance-based).

Points the reference leaves undefined, fixed here to the CUDA hardware result
so the GPU can be compared bit for bit: ``x // 0 = 0xFFFFFFFF``, ``x % 0 = x``;
float -> u32 casts truncate and saturate (NaN -> 0).

The interpreter is duck-typed: it reads ``ir.args`` / ``ir.insts`` and
``inst.op/out/args`` with dtypes compared by their string value, so it runs
both this repository's IR objects and the reference front end's own objects.
"""

from __future__ import annotations

import math
from typing import Any, Mapping

import numpy as np

F32, F64, F16, U32 = np.float32, np.float64, np.float16, np.uint32
MASK32 = 0xFFFFFFFF


class OracleError(RuntimeError):
    pass


def _dt(x: Any) -> str:
    return getattr(x, "value", x)


# ---------------------------------------------------------------------------
# exact arithmetic helpers
# ---------------------------------------------------------------------------


def fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Correctly rounded float32 ``a*b + c`` (round-to-nearest-even).

    ``a*b`` is exact in float64; ``s = p + c`` is computed with its exact
    error ``e`` (TwoSum).  ``RN32(p + c)`` equals ``RN32(s)`` unless ``s`` is
    exactly halfway between two float32 values, in which case the sign of
    ``e`` decides.
    """
    a, b, c = (np.asarray(x, dtype=F32) for x in (a, b, c))
    cc = c.astype(F64)
    with np.errstate(over="ignore", invalid="ignore"):
        p = a.astype(F64) * b.astype(F64)
        s = p + cc
        bb = s - p
        e = (p - (s - bb)) + (cc - bb)
        r = s.astype(F32)
        r64 = r.astype(F64)
        diff = s - r64
        toward = np.where(diff > 0, np.float32(np.inf), np.float32(-np.inf)).astype(F32)
        other = np.nextafter(r, toward)
        mid = (diff != 0) & np.isfinite(s) & (np.abs(other.astype(F64) - r64) == 2 * np.abs(diff))
        fix = mid & (e != 0) & (np.sign(e) == np.sign(diff))
    return np.where(fix, other, r).astype(F32)


def f2u(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=F64)
    with np.errstate(invalid="ignore"):
        t = np.trunc(np.nan_to_num(x, nan=0.0, posinf=float(MASK32), neginf=0.0))
    return np.clip(t, 0, MASK32).astype(np.uint64).astype(U32)


def cast(x: np.ndarray, src: str, dst: str) -> np.ndarray:
    if src == dst:
        return x
    if dst == "bool":
        return x.astype(F32) != 0 if src == "f16" else x != 0
    if src == "bool":
        return x.astype({"u32": U32, "f32": F32, "f16": F16}[dst])
    if dst == "u32":
        return f2u(x)
    if dst == "f32":
        return x.astype(F32)  # u32 -> f32 and f16 -> f32: single rounding / exact
    if dst == "f16":  # beyond the f16 range the round-to-nearest result is +-inf, as intended
        with np.errstate(over="ignore"):
            return x.astype(F64).astype(F16) if src == "u32" else x.astype(F32).astype(F16)
    raise OracleError(f"bad cast {src}->{dst}")


def arith(op: str, dt: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore", invalid="ignore"):
        if dt == "u32":
            a64, b64 = a.astype(np.uint64), b.astype(np.uint64)
            if op == "add":
                return ((a64 + b64) & MASK32).astype(U32)
            if op == "mul":
                return ((a64 * b64) & MASK32).astype(U32)
            safe = np.where(b64 == 0, 1, b64)
            if op == "floordiv":
                return np.where(b64 == 0, MASK32, a64 // safe).astype(U32)
            if op == "mod":
                return np.where(b64 == 0, a64, a64 % safe).astype(U32)
        af, bf = a.astype(F32), b.astype(F32)
        r = af + bf if op == "add" else af * bf
        return r.astype(F16) if dt == "f16" else r.astype(F32)
    raise OracleError(f"bad arith {op} {dt}")


# ---------------------------------------------------------------------------
# launch geometry (metal.py:257-326, grid.py)
# ---------------------------------------------------------------------------


def block_and_mode(ir: Any) -> tuple[int, str]:
    ar = {int(i.args[1]) for i in ir.insts if i.op == "arange"}
    td = {int(i.args[1]) for i in ir.insts if i.op == "tid"}
    if len(ar) > 1 or len(td) > 1 or (ar and td):
        raise OracleError("ambiguous block size / mode")
    if ar:
        return ar.pop(), "spmd"
    if td:
        return td.pop(), "thread"
    raise OracleError("kernel defines no BLOCK")


def geometry(ir: Any, runtime_args: Mapping[str, Any], *, nthreads: int | None = None,
             grid: tuple[int, ...] | None = None, shape: tuple[int, ...] | None = None
             ) -> tuple[int, str, tuple[int, int, int], int | None]:
    """(BLOCK, mode, programs per axis, exact thread count for 1D thread launches or None)."""
    block, mode = block_and_mode(ir)
    if grid is not None:
        g = tuple(int(x) for x in grid) + (1,) * (3 - len(grid))
        return block, mode, g, None  # type: ignore[return-value]
    rank = max([int(i.args[0]) for i in ir.insts if i.op in ("program_id", "thread_id")], default=-1) + 1
    if rank <= 1:
        n = int(nthreads) if nthreads is not None else int(runtime_args["N"])
        progs = math.ceil(n / block)
        return block, mode, (progs, 1, 1), (n if mode == "thread" else None)
    if shape is not None:
        dims = list(shape)
        h, w = dims[-2], dims[-1]
        d = dims[-3] if rank == 3 else 1
    else:
        h, w = int(runtime_args["H"]), int(runtime_args["W"])
        d = int(runtime_args["D"]) if rank == 3 else 1
    return block, mode, (math.ceil(w / block) if w else 0, h, d), None


# ---------------------------------------------------------------------------
# interpreter
# ---------------------------------------------------------------------------

_NP = {"f32": F32, "f16": F16, "u32": U32, "bool": np.bool_}


class _Machine:
    """Executes one launch for all programs/threads in lockstep."""

    def __init__(self, ir: Any, buffers: dict[str, np.ndarray], scalars: dict[str, Any], block: int, mode: str,
                 programs: tuple[int, int, int], n_threads_1d: int | None,
                 pid_base: tuple[int, int, int] = (0, 0, 0)):
        self.ir, self.buffers, self.scalars = ir, buffers, scalars
        self.block, self.mode = block, mode
        gx, gy, gz = programs
        bx, by, bz = (int(b) for b in pid_base)
        self.P = gx * gy * gz
        pid = np.arange(self.P, dtype=np.int64)
        self.pid = ((pid % gx + bx).astype(U32), ((pid // gx) % gy + by).astype(U32),
                    (pid // (gx * gy) + bz).astype(U32))
        if mode == "thread":
            # threads: (program, local) pairs; a 1D launch of exactly n threads drops the tail of the last group
            loc = np.tile(np.arange(block, dtype=np.int64), self.P)
            grp = np.repeat(np.arange(self.P, dtype=np.int64), block)
            if n_threads_1d is not None:
                keep = (grp + bx) * block + loc < n_threads_1d   # global thread index, as on the device
                loc, grp = loc[keep], grp[keep]
            self.loc, self.grp = loc, grp
            self.shape = (len(loc),)
        else:
            self.shape = (self.P, 1)
        self.vals: dict[int, Any] = {}
        self.tg: dict[int, np.ndarray] = {}
        self.buf_of: dict[int, tuple[str, Any]] = {}

    # -- value access ---------------------------------------------------------
    def get(self, ref: Any) -> Any:
        return self.vals[ref.id]

    def bcast(self, x: np.ndarray) -> np.ndarray:
        return x

    # -- memory -------------------------------------------------------------------
    def _addr(self, buf_ref: Any, off: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """(flat storage, flat index array) for a buffer access."""
        kind, key = self.buf_of[buf_ref.id]
        off = off.astype(np.int64)
        if kind == "arg":
            return self.buffers[key].reshape(-1), off
        store = self.tg[key]  # (P, size)
        size = store.shape[1]
        if self.mode == "thread":
            grp = self.grp
        else:
            grp = np.arange(self.P, dtype=np.int64)[:, None]
        return store.reshape(-1), grp * size + off

    def load(self, buf_ref: Any, off: np.ndarray, mask: np.ndarray, dt: str) -> np.ndarray:
        mem, idx = self._addr(buf_ref, off)
        idx, mask = np.broadcast_arrays(idx, mask)
        out = np.zeros(idx.shape, dtype=_NP[dt])
        m = mask.astype(bool)
        sel = idx[m]
        if sel.size and (sel.min() < 0 or sel.max() >= mem.size):
            raise OracleError(f"out-of-bounds load from {self.buf_of[buf_ref.id][1]!r}: index {sel.max()}")
        out[m] = mem[sel]
        return out

    def store(self, buf_ref: Any, off: np.ndarray, val: np.ndarray, mask: np.ndarray) -> None:
        mem, idx = self._addr(buf_ref, off)
        idx, val, mask = np.broadcast_arrays(idx, val, mask)
        m = mask.astype(bool)
        sel = idx[m]
        if sel.size and (sel.min() < 0 or sel.max() >= mem.size):
            raise OracleError(f"out-of-bounds store to {self.buf_of[buf_ref.id][1]!r}: index {sel.max()}")
        mem[sel] = val[m].astype(mem.dtype)

    # -- per-thread ids (thread mode) ---------------------------------------------
    def pid_of(self, axis: int) -> np.ndarray:
        p = self.pid[axis]
        return p[self.grp] if self.mode == "thread" else p[:, None]

    def run(self) -> None:
        for inst in self.ir.insts:
            self.step(inst)

    def step(self, inst: Any) -> None:
        op, out, a = inst.op, inst.out, inst.args
        V = self.vals
        if op == "arg":
            name = str(a[0])
            if a[1] == "buffer":
                self.buf_of[out.id] = ("arg", name)
                V[out.id] = None
            else:
                V[out.id] = np.full(self.shape, self.scalars[name], dtype=_NP[_dt(out.dtype)])
        elif op == "const":
            v = a[0]
            dt = _dt(out.dtype)
            if dt == "u32":
                v = int(v) & MASK32
            elif dt == "f32":
                v = np.float32(v)
            V[out.id] = np.full(self.shape, v, dtype=_NP[dt])
        elif op == "alloc_tg":
            dt = _dt(out.dtype)
            self.tg[out.id] = np.zeros((self.P, int(a[0])), dtype=_NP[dt])
            self.buf_of[out.id] = ("tg", out.id)
            V[out.id] = None
        elif op == "program_id":
            V[out.id] = self.pid_of(int(a[0]))
        elif op == "thread_id":
            ax = int(a[0])
            if self.mode == "thread" and ax == 0:
                V[out.id] = (self.pid[0][self.grp].astype(np.int64) * self.block + self.loc).astype(U32)
            else:
                V[out.id] = self.pid_of(ax)
        elif op == "local_id":
            V[out.id] = self.loc.astype(U32) if int(a[0]) == 0 else np.zeros(self.shape, U32)
        elif op == "lane_id":
            V[out.id] = (self.loc % 32).astype(U32)
        elif op == "sg_id":
            V[out.id] = (self.loc // 32).astype(U32)
        elif op == "tid":
            V[out.id] = (int(a[0]) + self.loc).astype(U32)
        elif op == "arange":
            start, size = int(a[0]), int(a[1])
            V[out.id] = np.broadcast_to((start + np.arange(size, dtype=np.int64)).astype(U32), (self.P, size))
        elif op in ("add", "mul", "floordiv", "mod"):
            V[out.id] = arith(op, _dt(a[0].dtype), self.get(a[0]), self.get(a[1]))
        elif op == "lt":
            x, y = self.get(a[0]), self.get(a[1])
            if _dt(a[0].dtype) == "f16":
                x, y = x.astype(F32), y.astype(F32)
            V[out.id] = x < y
        elif op == "and":
            V[out.id] = np.logical_and(self.get(a[0]), self.get(a[1]))
        elif op == "or":
            V[out.id] = np.logical_or(self.get(a[0]), self.get(a[1]))
        elif op == "not":
            V[out.id] = np.logical_not(self.get(a[0]))
        elif op == "where":
            V[out.id] = np.where(self.get(a[0]), self.get(a[1]), self.get(a[2])).astype(_NP[_dt(out.dtype)])
        elif op == "cast":
            V[out.id] = cast(self.get(a[0]), _dt(a[0].dtype), _dt(a[1]))
        elif op == "fma":
            r = fma_f32(*(self.get(x).astype(F32) for x in a))
            V[out.id] = r.astype(F16) if _dt(out.dtype) == "f16" else r
        elif op == "load":
            V[out.id] = self.load(a[0], self.get(a[1]), self.get(a[2]), _dt(out.dtype))
        elif op == "store":
            self.store(a[0], self.get(a[1]), self.get(a[2]), self.get(a[3]))
        elif op == "barrier":
            pass
        elif op == "dot":
            self._dot(inst)
        elif op == "mma_zero":
            V[out.id] = np.zeros(self.shape + (8, 8), dtype=F32)
        elif op == "mma":
            self._mma(inst)
        elif op == "mma_store":
            self._mma_store(inst)
        else:
            raise OracleError(f"unsupported op {op!r}")

    def _dot(self, inst: Any) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, k = inst.args
        ab = self.get(a_base).astype(np.uint64)
        bb = self.get(b_base).astype(np.uint64)
        sa = self.get(a_stride).astype(np.uint64)
        sb = self.get(b_stride).astype(np.uint64)
        K = self.get(k).astype(np.int64)
        acc = np.zeros(self.shape, dtype=F32)
        kmax = int(K.max()) if K.size else 0
        true = np.ones(self.shape, dtype=bool)
        for kk in range(kmax):
            active = K > kk
            ai = ((ab + sa * np.uint64(kk)) & MASK32).astype(U32)
            bi = ((bb + sb * np.uint64(kk)) & MASK32).astype(U32)
            av = self.load(a_buf, ai, active & true, _dt(a_buf.dtype)).astype(F32)
            bv = self.load(b_buf, bi, active & true, _dt(b_buf.dtype)).astype(F32)
            acc = np.where(active, fma_f32(av, bv, acc), acc)
        self.vals[inst.out.id] = acc

    def _sg_first(self) -> tuple[np.ndarray, np.ndarray]:
        """Index of each thread's simdgroup leader, and of the leaders themselves."""
        key = self.grp * ((self.block + 31) // 32) + self.loc // 32
        _, first, inv = np.unique(key, return_index=True, return_inverse=True)
        return first, inv

    def _tile(self, buf_ref: Any, base: np.ndarray, stride: np.ndarray, leaders: np.ndarray) -> np.ndarray:
        r = np.arange(8, dtype=np.int64)
        off = (base[leaders].astype(np.int64)[:, None, None]
               + r[None, :, None] * stride[leaders].astype(np.int64)[:, None, None] + r[None, None, :]) & MASK32
        kind, key = self.buf_of[buf_ref.id]
        if kind == "arg":
            mem, idx = self.buffers[key].reshape(-1), off
        else:
            mem = self.tg[key].reshape(-1)
            idx = self.grp[leaders][:, None, None] * self.tg[key].shape[1] + off
        if idx.size and (idx.min() < 0 or idx.max() >= mem.size):
            raise OracleError("out-of-bounds mma tile access")
        return mem[idx].astype(F64)

    def _mma(self, inst: Any) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, acc = inst.args
        first, inv = self._sg_first()
        A = self._tile(a_buf, self.get(a_base), self.get(a_stride), first)
        B = self._tile(b_buf, self.get(b_base), self.get(b_stride), first)
        C = self.get(acc)[first].astype(F64)
        D = (A @ B + C).astype(F32)
        self.vals[inst.out.id] = D[inv]

    def _mma_store(self, inst: Any) -> None:
        buf, base, stride, frag = inst.args
        first, _inv = self._sg_first()
        D = self.get(frag)[first]
        r = np.arange(8, dtype=np.int64)
        off = (self.get(base)[first].astype(np.int64)[:, None, None]
               + r[None, :, None] * self.get(stride)[first].astype(np.int64)[:, None, None] + r[None, None, :])
        kind, key = self.buf_of[buf.id]
        if kind == "arg":
            mem = self.buffers[key].reshape(-1)
            idx = off
        else:
            mem = self.tg[key].reshape(-1)
            idx = self.grp[first][:, None, None] * self.tg[key].shape[1] + off
        if idx.size and (idx.min() < 0 or idx.max() >= mem.size):
            raise OracleError("out-of-bounds mma_store")
        mem[idx.reshape(-1)] = D.reshape(-1)


def execute(ir: Any, runtime_args: Mapping[str, Any], *, nthreads: int | None = None,
            grid: tuple[int, ...] | None = None, shape: tuple[int, ...] | None = None,
            pid_base: tuple[int, int, int] = (0, 0, 0), ntx: int | None = None) -> None:
    """Run ``ir`` once on the CPU.  Buffers are numpy arrays, updated in place.

    ``pid_base`` and ``ntx`` describe one launch of a split grid, as the generated kernel's hidden
    parameters do: program ids start at ``pid_base``, and in thread mode only global threads below
    ``ntx`` run."""
    block, mode, programs, n1d = geometry(ir, runtime_args, nthreads=nthreads, grid=grid, shape=shape)
    if ntx is not None and mode == "thread":
        n1d = int(ntx)
    if min(programs) == 0 or (n1d is not None and n1d == 0):
        return
    buffers: dict[str, np.ndarray] = {}
    scalars: dict[str, Any] = {}
    for arg in ir.args:
        v = runtime_args[arg.name]
        if arg.kind == "buffer":
            if not isinstance(v, np.ndarray) or not v.flags.c_contiguous:
                raise OracleError(f"buffer {arg.name!r} must be a C-contiguous numpy array")
            buffers[arg.name] = v
        else:
            scalars[arg.name] = v
    _Machine(ir, buffers, scalars, block, mode, programs, n1d, pid_base).run()
