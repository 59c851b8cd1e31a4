"""Tracer and IR optimisation passes.

``trace_to_ir`` runs a kernel's Python body once, with every runtime argument
replaced by a traced :class:`~easy_as_b200.mk.val`; each ``mk.*`` call appends
one SSA instruction.  The passes then rewrite the flat instruction list.

Both follow the reference front end exactly, because the IR they produce is
the contract the CUDA emitter, the CPU oracle and the golden fixtures share:

* argument typing and value numbering: easy_as ``eas/compiler.py:57-129,132-550``
* ``trace_to_ir`` / meta-as-globals: ``eas/compiler.py:553-617``
* pass order: ``eas/compiler.py:648-655``
  (thread-id rewrite ``:937-1016``, FMA fusion ``:1019-1096``, interval ``lt``
  folding ``:658-795``, bool simplification ``:798-934``, CSE ``:1099-1200``,
  DCE ``:1203-1272``).

The golden fixtures under ``tests/golden`` hold IR produced by the reference
front end for a set of kernels; the tests require this module to reproduce
them instruction for instruction.
"""

from __future__ import annotations

import os
import types
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping

import numpy as np

from . import mk
from .analysis import infer_writes
from .ir import Arg, ArgKind, DType, IRModule, Inst, SIDE_EFFECT_OPS, ValueRef, validate_ir
from .tensor import Tensor as _Tensor

# ---------------------------------------------------------------------------
# argument classification
# ---------------------------------------------------------------------------

_torch_mod: Any = None
_torch_probed = False


def _torch() -> Any:
    global _torch_mod, _torch_probed
    if not _torch_probed:
        _torch_probed = True
        try:
            import torch  # type: ignore

            _torch_mod = torch
        except Exception:
            _torch_mod = None
    return _torch_mod


def _is_eas_tensor(v: Any) -> bool:
    return bool(getattr(v, "__eas_tensor__", False))


def _is_torch_tensor(v: Any) -> bool:
    t = _torch()
    return t is not None and isinstance(v, t.Tensor)


def is_buffer_value(v: Any) -> bool:
    return isinstance(v, np.ndarray) or _is_eas_tensor(v) or _is_torch_tensor(v)


def _float_dtype(np_dtype: Any, what: str) -> DType:
    d = np.dtype(np_dtype)
    if d == np.float32:
        return DType.F32
    if d == np.float16:
        return DType.F16
    raise TypeError(f"unsupported {what}dtype: {np_dtype} (expected float32 or float16)")


def buffer_dtype(v: Any) -> DType:
    if isinstance(v, np.ndarray):
        return _float_dtype(v.dtype, "")
    if _is_torch_tensor(v):
        t = _torch()
        table = {t.float32: DType.F32, t.float16: DType.F16}
        if v.dtype not in table:
            raise TypeError(f"unsupported torch dtype: {v.dtype} (expected float32 or float16)")
        return table[v.dtype]
    dt = getattr(v, "dtype", None)
    if dt is None:
        raise TypeError("tensor argument is missing dtype")
    return _float_dtype(dt, "tensor ")


def scalar_dtype(v: Any) -> DType:
    if isinstance(v, (bool, np.bool_)):
        return DType.BOOL
    if isinstance(v, (int, np.integer)):
        return DType.U32
    if isinstance(v, np.float16):
        return DType.F16
    if isinstance(v, (float, np.floating)):
        return DType.F32
    raise TypeError(f"unsupported scalar type: {type(v)!r}")


@dataclass(frozen=True, slots=True)
class RuntimeArgSig:
    kind: ArgKind
    dtype: DType
    device: str | None = None


def _arg_sig(v: Any) -> RuntimeArgSig:
    if isinstance(v, np.ndarray):
        return RuntimeArgSig("buffer", buffer_dtype(v), "cpu")
    if _is_eas_tensor(v):
        dev = getattr(v, "device", None)
        return RuntimeArgSig("buffer", buffer_dtype(v), str(dev) if dev else None)
    if _is_torch_tensor(v):
        try:
            return RuntimeArgSig("buffer", buffer_dtype(v), str(v.device.type))
        except Exception:
            return RuntimeArgSig("buffer", DType.F32, None)
    return RuntimeArgSig("scalar", scalar_dtype(v), None)


_SCALAR_SIGS = {bool: ("scalar", DType.BOOL, None), int: ("scalar", DType.U32, None),
                float: ("scalar", DType.F32, None)}


_TENSOR_DTYPES = {np.dtype(np.float32): DType.F32, np.dtype(np.float16): DType.F16}


def fast_arg_sig(v: Any) -> tuple[Any, ...]:
    """(kind, dtype, device) of one runtime argument; the launch-path form of ``_arg_sig``."""
    s = _SCALAR_SIGS.get(type(v))
    if s is not None:
        return s
    if type(v) is _Tensor:   # eas.Tensor: dtype and device are fixed at construction
        return ("buffer", _TENSOR_DTYPES[v._dtype], v._device)
    if type(v) is np.ndarray:
        dt = _TENSOR_DTYPES.get(v.dtype)
        if dt is not None:
            return ("buffer", dt, "cpu")
    t = _torch()
    if t is not None and isinstance(v, t.Tensor):
        dev = "cuda" if v.is_cuda else v.device.type
        if v.dtype == t.float32:
            return ("buffer", DType.F32, dev)
        if v.dtype == t.float16:
            return ("buffer", DType.F16, dev)
    sig = _arg_sig(v)
    return (sig.kind, sig.dtype, sig.device)


def runtime_arg_signature(runtime_args: Mapping[str, Any]) -> tuple[tuple[str, Any], ...]:
    """Cache key part for runtime arguments: kinds/dtypes/devices, never scalar values."""
    return tuple(sorted((name, (s.kind, s.dtype, s.device))
                        for name, s in ((n, _arg_sig(v)) for n, v in runtime_args.items())))


# ---------------------------------------------------------------------------
# tracer
# ---------------------------------------------------------------------------


class _Tracer:
    """Receives ``mk.*`` calls and appends SSA instructions."""

    def __init__(self, name: str) -> None:
        self.name = name
        self.args: list[Arg] = []
        self.insts: list[Inst] = []
        self.buffer_ids: set[int] = set()
        self.next_id = 0

    # -- value construction -------------------------------------------------
    def fresh(self, dtype: DType, lanes: int = 1) -> mk.val:
        v = mk.val(ValueRef(self.next_id, dtype, int(lanes)))
        self.next_id += 1
        return v

    def emit(self, op: str, dtype: DType | None, args: tuple[Any, ...], lanes: int = 1) -> mk.val | None:
        if dtype is None:
            self.insts.append(Inst(op, None, args))  # type: ignore[arg-type]
            return None
        out = self.fresh(dtype, lanes)
        self.insts.append(Inst(op, out.ref, args))  # type: ignore[arg-type]
        return out

    def lit(self, x: Any) -> mk.val:
        if isinstance(x, mk.val):
            return x
        if isinstance(x, bool):
            return self.emit("const", DType.BOOL, (bool(x),))  # type: ignore[return-value]
        if isinstance(x, (int, np.integer)):
            return self.emit("const", DType.U32, (int(x),))  # type: ignore[return-value]
        if isinstance(x, (float, np.floating)):
            return self.emit("const", DType.F32, (float(x),))  # type: ignore[return-value]
        raise TypeError(f"unsupported literal: {type(x)!r}")

    @staticmethod
    def _pair_lanes(op: str, a: mk.val, b: mk.val) -> int:
        la, lb = a.ref.lanes, b.ref.lanes
        if la != lb and la != 1 and lb != 1:
            raise TypeError(f"{op} lanes mismatch: {la} vs {lb}")
        return lb if la == 1 else la

    def _binary(self, op: str, a: Any, b: Any, *, out_dtype: DType | None = None,
                need: DType | None = None, bool_ops: bool = False) -> mk.val:
        av, bv = self.lit(a), self.lit(b)
        if bool_ops:
            if av.dtype != DType.BOOL or bv.dtype != DType.BOOL:
                raise TypeError("and/or/not expect bool operands")
        else:
            if av.dtype != bv.dtype:
                raise TypeError(f"{op} dtype mismatch: {av.dtype} vs {bv.dtype}")
            if need is not None and av.dtype != need:
                raise TypeError(f"{op} expects u32, got {av.dtype}")
        lanes = self._pair_lanes(op, av, bv)
        ir_op = {"and_": "and", "or_": "or"}.get(op, op)
        return self.emit(ir_op, out_dtype or av.dtype, (av.ref, bv.ref), lanes)  # type: ignore[return-value]

    # -- ids ------------------------------------------------------------------
    def program_id(self, axis: int) -> mk.val:
        return self.emit("program_id", DType.U32, (int(axis),))  # type: ignore[return-value]

    def local_id(self, axis: int) -> mk.val:
        if not isinstance(axis, int):
            raise TypeError("local_id(axis) requires an int axis")
        if axis not in (0, 1, 2):
            raise ValueError("local_id axis must be 0/1/2")
        return self.emit("local_id", DType.U32, (axis,))  # type: ignore[return-value]

    def lane_id(self) -> mk.val:
        return self.emit("lane_id", DType.U32, ())  # type: ignore[return-value]

    def sg_id(self) -> mk.val:
        return self.emit("sg_id", DType.U32, ())  # type: ignore[return-value]

    def _range_args(self, what: str, start: Any, size: Any) -> tuple[int, int]:
        if not isinstance(start, int) or not isinstance(size, int):
            raise TypeError(f"{what}(start, size) requires Python ints (compile-time constants)")
        if size <= 0:
            raise ValueError(f"{what}(size) must be > 0")
        return int(start), int(size)

    def arange(self, start: int, size: int) -> mk.val:
        s, n = self._range_args("arange", start, size)
        return self.emit("arange", DType.U32, (s, n), lanes=n)  # type: ignore[return-value]

    def tid(self, start: int, size: int) -> mk.val:
        s, n = self._range_args("tid", start, size)
        return self.emit("tid", DType.U32, (s, n))  # type: ignore[return-value]

    def alloc_tg(self, size: int, *, dtype: DType = DType.F32) -> mk.val:
        if not isinstance(size, int):
            raise TypeError("alloc_tg(size) requires a Python int (compile-time constant)")
        if size <= 0:
            raise ValueError("alloc_tg(size) must be > 0")
        if dtype not in (DType.F16, DType.F32):
            raise TypeError(f"alloc_tg(dtype=...) must be f16/f32, got {dtype}")
        v = self.emit("alloc_tg", dtype, (int(size),))
        assert v is not None
        self.buffer_ids.add(v.ref.id)
        return v

    def barrier(self) -> None:
        self.emit("barrier", None, ())

    # -- arithmetic -------------------------------------------------------------
    def add(self, a: Any, b: Any) -> mk.val:
        return self._binary("add", a, b)

    def mul(self, a: Any, b: Any) -> mk.val:
        return self._binary("mul", a, b)

    def floordiv(self, a: Any, b: Any) -> mk.val:
        return self._binary("floordiv", a, b, need=DType.U32)

    def mod(self, a: Any, b: Any) -> mk.val:
        return self._binary("mod", a, b, need=DType.U32)

    def lt(self, a: Any, b: Any) -> mk.val:
        return self._binary("lt", a, b, out_dtype=DType.BOOL)

    def and_(self, a: Any, b: Any) -> mk.val:
        return self._binary("and_", a, b, out_dtype=DType.BOOL, bool_ops=True)

    def or_(self, a: Any, b: Any) -> mk.val:
        return self._binary("or_", a, b, out_dtype=DType.BOOL, bool_ops=True)

    def not_(self, x: Any) -> mk.val:
        xv = self.lit(x)
        if xv.dtype != DType.BOOL:
            raise TypeError("and/or/not expect bool operands")
        return self.emit("not", DType.BOOL, (xv.ref,), xv.ref.lanes)  # type: ignore[return-value]

    def fma(self, a: Any, b: Any, c: Any) -> mk.val:
        vals = [self.lit(a), self.lit(b), self.lit(c)]
        if len({v.dtype for v in vals}) != 1:
            raise TypeError(f"fma dtype mismatch: {vals[0].dtype} vs {vals[1].dtype} vs {vals[2].dtype}")
        lanes = vals[0].ref.lanes
        for v in vals[1:]:
            if lanes == 1:
                lanes = v.ref.lanes
            elif v.ref.lanes not in (1, lanes):
                raise TypeError(f"fma lanes mismatch: {lanes} vs {v.ref.lanes}")
        return self.emit("fma", vals[0].dtype, tuple(v.ref for v in vals), lanes)  # type: ignore[return-value]

    def where(self, cond: Any, a: Any, b: Any) -> mk.val:
        cv, av, bv = self.lit(cond), self.lit(a), self.lit(b)
        if cv.dtype != DType.BOOL:
            raise TypeError(f"where(cond, ...) expects bool condition, got {cv.dtype}")
        if av.dtype != bv.dtype:
            raise TypeError(f"where value dtype mismatch: {av.dtype} vs {bv.dtype}")
        lanes = next((v.ref.lanes for v in (av, bv, cv) if v.ref.lanes != 1), 1)
        for v in (bv, cv):
            if v.ref.lanes not in (1, lanes):
                raise TypeError(f"where lanes mismatch: {lanes} vs {v.ref.lanes}")
        return self.emit("where", av.dtype, (cv.ref, av.ref, bv.ref), lanes)  # type: ignore[return-value]

    def cast(self, x: Any, dtype: DType) -> mk.val:
        xv = self.lit(x)
        if not isinstance(dtype, DType):
            raise TypeError("cast(x, dtype) expects dtype to be a DType")
        if xv.dtype == dtype:
            return xv
        return self.emit("cast", dtype, (xv.ref, dtype), xv.ref.lanes)  # type: ignore[return-value]

    # -- memory -------------------------------------------------------------------
    def _need_buffer(self, x: Any, msg: str) -> mk.val:
        if not isinstance(x, mk.val) or x.ref.id not in self.buffer_ids:
            raise TypeError(msg)
        return x

    def load(self, buffer: Any, offset: Any, mask: Any | None) -> mk.val:
        buf = self._need_buffer(buffer, "load(buffer, ...) expects a buffer (arg or alloc_tg)")
        off = self.lit(offset)
        m = self.lit(True if mask is None else mask)
        if off.dtype != DType.U32:
            raise TypeError(f"load offset must be u32, got {off.dtype}")
        if m.dtype != DType.BOOL:
            raise TypeError(f"load mask must be bool, got {m.dtype}")
        if m.ref.lanes not in (1, off.ref.lanes):
            raise TypeError(f"load mask lanes must be 1 or match offset lanes, got {m.ref.lanes} vs {off.ref.lanes}")
        return self.emit("load", buf.dtype, (buf.ref, off.ref, m.ref), off.ref.lanes)  # type: ignore[return-value]

    def store(self, buffer: Any, offset: Any, value: Any, mask: Any | None) -> None:
        buf = self._need_buffer(buffer, "store(buffer, ...) expects a buffer (arg or alloc_tg)")
        off = self.lit(offset)
        v = self.lit(value)
        m = self.lit(True if mask is None else mask)
        if off.dtype != DType.U32:
            raise TypeError(f"store offset must be u32, got {off.dtype}")
        if m.dtype != DType.BOOL:
            raise TypeError(f"store mask must be bool, got {m.dtype}")
        if v.dtype != buf.dtype:
            raise TypeError(f"store dtype mismatch: {buf.dtype} vs {v.dtype}")
        for what, x in (("value", v), ("mask", m)):
            if x.ref.lanes not in (1, off.ref.lanes):
                raise TypeError(f"store {what} lanes must be 1 or match offset lanes, "
                                f"got {x.ref.lanes} vs {off.ref.lanes}")
        self.emit("store", None, (buf.ref, off.ref, v.ref, m.ref))

    def _index_operands(self, op: str, named: list[tuple[str, Any]]) -> list[mk.val]:
        out = []
        for name, x in named:
            v = self.lit(x)
            if v.dtype != DType.U32:
                raise TypeError(f"{op} {name} must be u32, got {v.dtype}")
            if v.ref.lanes != 1:
                raise TypeError(f"{op} {name} must be scalar (lanes=1), got lanes={v.ref.lanes}")
            out.append(v)
        return out

    def dot(self, a_buffer: Any, a_base: Any, a_stride: Any, b_buffer: Any, b_base: Any,
            b_stride: Any, K: Any) -> mk.val:
        a = self._need_buffer(a_buffer, "dot expects a_buffer to be a buffer (arg or alloc_tg)")
        b = self._need_buffer(b_buffer, "dot expects b_buffer to be a buffer (arg or alloc_tg)")
        if a.dtype not in (DType.F16, DType.F32):
            raise TypeError("dot a_buffer must be f16/f32")
        if b.dtype not in (DType.F16, DType.F32):
            raise TypeError("dot b_buffer must be f16/f32")
        ab, ast, bb, bst, k = self._index_operands("dot", [
            ("a_base", a_base), ("a_stride", a_stride), ("b_base", b_base), ("b_stride", b_stride), ("K", K)])
        return self.emit("dot", DType.F32, (a.ref, ab.ref, ast.ref, b.ref, bb.ref, bst.ref, k.ref))  # type: ignore[return-value]

    def mma_zero(self) -> mk.val:
        return self.emit("mma_zero", DType.SG_F32_8X8, ())  # type: ignore[return-value]

    def mma(self, a_buffer: Any, a_base: Any, a_stride: Any, b_buffer: Any, b_base: Any,
            b_stride: Any, acc: Any) -> mk.val:
        a = self._need_buffer(a_buffer, "mma expects a_buffer to be a buffer (arg or alloc_tg)")
        b = self._need_buffer(b_buffer, "mma expects b_buffer to be a buffer (arg or alloc_tg)")
        if a.dtype not in (DType.F16, DType.F32) or b.dtype not in (DType.F16, DType.F32):
            raise TypeError("mma currently supports f16/f32 buffers only")
        ab, ast, bb, bst = self._index_operands("mma", [
            ("a_base", a_base), ("a_stride", a_stride), ("b_base", b_base), ("b_stride", b_stride)])
        accv = self.lit(acc)
        if accv.dtype != DType.SG_F32_8X8:
            raise TypeError(f"mma acc must be sg_f32_8x8, got {accv.dtype}")
        if accv.ref.lanes != 1:
            raise TypeError(f"mma acc must be scalar (lanes=1), got lanes={accv.ref.lanes}")
        return self.emit("mma", DType.SG_F32_8X8,  # type: ignore[return-value]
                         (a.ref, ab.ref, ast.ref, b.ref, bb.ref, bst.ref, accv.ref))

    def mma_store(self, buffer: Any, base: Any, stride: Any, frag: Any) -> None:
        buf = self._need_buffer(buffer, "mma_store(buffer, ...) expects a buffer (arg or alloc_tg)")
        if buf.dtype != DType.F32:
            raise TypeError("mma_store currently supports float32 buffers only")
        bv, sv, fv = self.lit(base), self.lit(stride), self.lit(frag)
        if bv.dtype != DType.U32:
            raise TypeError(f"mma_store base must be u32, got {bv.dtype}")
        if sv.dtype != DType.U32:
            raise TypeError(f"mma_store stride must be u32, got {sv.dtype}")
        if fv.dtype != DType.SG_F32_8X8:
            raise TypeError(f"mma_store frag must be sg_f32_8x8, got {fv.dtype}")
        if bv.ref.lanes != 1 or sv.ref.lanes != 1 or fv.ref.lanes != 1:
            raise TypeError("mma_store base/stride/frag must be scalar (lanes=1)")
        self.emit("mma_store", None, (buf.ref, bv.ref, sv.ref, fv.ref))


def _bind_meta_globals(fn: Callable[..., Any], meta: Mapping[str, Any]) -> Callable[..., Any]:
    """Copy of ``fn`` whose globals also see the constexpr parameters."""
    if not meta:
        return fn
    g = dict(fn.__globals__)
    g.update(meta)
    return types.FunctionType(fn.__code__, g, name=fn.__name__, argdefs=fn.__defaults__,
                              closure=fn.__closure__)


def trace_to_ir(fn: Callable[..., Any], runtime_args: Mapping[str, Any], meta: Mapping[str, Any]) -> IRModule:
    tr = _Tracer(fn.__name__)
    kwargs: dict[str, Any] = {}
    for name, value in runtime_args.items():
        if is_buffer_value(value):
            arg = Arg(name, buffer_dtype(value), "buffer")
        else:
            arg = Arg(name, scalar_dtype(value), "scalar")
        tr.args.append(arg)
        v = tr.emit("arg", arg.dtype, (name, arg.kind, arg.dtype))
        assert v is not None
        if arg.kind == "buffer":
            tr.buffer_ids.add(v.ref.id)
        kwargs[name] = v
    for name, value in meta.items():
        if isinstance(value, np.integer):
            value = int(value)
        elif isinstance(value, np.floating):
            value = float(value)
        if not isinstance(value, (bool, int, float)):
            raise TypeError(f"meta parameter {name!r} must be a Python literal, got {type(value)!r}")
        kwargs[name] = value
    with mk._trace(tr):
        _bind_meta_globals(fn, meta)(**kwargs)
    return IRModule(fn.__name__, tuple(tr.args), tuple(tr.insts))


# ---------------------------------------------------------------------------
# compiled kernel
# ---------------------------------------------------------------------------


@dataclass(frozen=True, slots=True)
class CompiledKernel:
    """Result of tracing + optimising + lowering one specialisation.

    ``src`` is the generated CUDA C++ (``msl`` is kept as an alias of the
    reference's field name); ``plan`` describes how the runtime launches it
    (generic NVRTC module, or a pattern-lowered native kernel).
    """

    ir: IRModule
    src: str
    block_size: int
    launch_mode: str
    writes: frozenset[str]
    plan: Any = field(default=None, compare=False)

    @property
    def msl(self) -> str:
        return self.src

    @property
    def cuda(self) -> str:
        return self.src


def compile(fn: Callable[..., Any], runtime_args: Mapping[str, Any], meta: Mapping[str, Any]) -> CompiledKernel:
    ir = optimize_ir(trace_to_ir(fn, runtime_args, meta))
    validate_ir(ir)
    from .codegen.cuda import ir_to_cuda

    lowered = ir_to_cuda(ir)
    hints = getattr(getattr(lowered, "native", None), "apply_tile_hints", None)
    if hints is not None:
        hints(meta)
    return CompiledKernel(ir=ir, src=lowered.src, block_size=lowered.block_size,
                          launch_mode=lowered.mode, writes=infer_writes(ir), plan=lowered)


# ---------------------------------------------------------------------------
# passes
# ---------------------------------------------------------------------------


def optimize_ir(ir: IRModule) -> IRModule:
    for p in (_rewrite_thread_id, _fuse_fma, _fold_static_lts, _simplify_bools, _cse_pure, _dce):
        ir = p(ir)
    return ir


_optimize_ir = optimize_ir


def _defs(ir: IRModule) -> dict[int, Inst]:
    return {i.out.id: i for i in ir.insts if i.out is not None}


def _single_tid_size(ir: IRModule) -> int | None:
    """Threads per block when every ``tid`` agrees on it, else None."""
    sizes = {int(i.args[1]) for i in ir.insts if i.op == "tid"}
    return sizes.pop() if len(sizes) == 1 else None


def _remapper(table: dict[int, ValueRef]) -> Callable[[tuple[Any, ...]], tuple[Any, ...]]:
    return lambda args: tuple(table.get(a.id, a) if isinstance(a, ValueRef) else a for a in args)


def _rewrite_thread_id(ir: IRModule) -> IRModule:
    """``program_id(0) * NT + tid(0, NT)`` -> ``thread_id(0)`` (reference ``compiler.py:937-1016``).

    Disabled by ``EAS_DISABLE_THREAD_ID_REWRITE`` (any value but "", "0",
    "false", "False") and when tid sizes disagree.
    """
    if os.environ.get("EAS_DISABLE_THREAD_ID_REWRITE", "") not in ("", "0", "false", "False"):
        return ir
    if any(i.op == "tid" for i in ir.insts) and _single_tid_size(ir) is None:
        return ir
    nt = _single_tid_size(ir)
    if nt is None:
        return ir
    defs = _defs(ir)

    def op_of(ref: Any) -> Inst | None:
        return defs.get(ref.id) if isinstance(ref, ValueRef) else None

    def is_pid0(ref: Any) -> bool:
        d = op_of(ref)
        return d is not None and d.op == "program_id" and int(d.args[0]) == 0

    def is_nt(ref: Any) -> bool:
        d = op_of(ref)
        return d is not None and d.op == "const" and isinstance(d.args[0], int) and int(d.args[0]) == nt

    def block_base_plus_tid(m: Any, t: Any) -> bool:
        dm, dt = op_of(m), op_of(t)
        if dm is None or dt is None or dm.op != "mul" or dt.op != "tid":
            return False
        if (int(dt.args[0]), int(dt.args[1])) != (0, nt):
            return False
        x, y = dm.args
        if not (isinstance(x, ValueRef) and isinstance(y, ValueRef)):
            return False
        return (is_pid0(x) and is_nt(y)) or (is_pid0(y) and is_nt(x))

    out: list[Inst] = []
    for inst in ir.insts:
        if inst.op == "add" and inst.out is not None:
            a, b = inst.args
            if isinstance(a, ValueRef) and isinstance(b, ValueRef) and (
                    block_base_plus_tid(a, b) or block_base_plus_tid(b, a)):
                out.append(Inst("thread_id", inst.out, (0,)))
                continue
        out.append(inst)
    return IRModule(ir.name, ir.args, tuple(out))


def _fuse_fma(ir: IRModule) -> IRModule:
    """f32 ``add(mul(x, y), z)`` -> ``fma(x, y, z)`` when the mul has one use.

    The mul is looked for in the first add operand, then the second; only the
    first mul found is considered (reference ``compiler.py:1019-1096``).
    """
    defs = _defs(ir)
    uses: dict[int, int] = {}
    for inst in ir.insts:
        for a in inst.args:
            if isinstance(a, ValueRef):
                uses[a.id] = uses.get(a.id, 0) + 1

    fused_muls: set[int] = set()
    out: list[Inst] = []
    for inst in ir.insts:
        if inst.op == "add" and inst.out is not None:
            a, b = inst.args
            if isinstance(a, ValueRef) and isinstance(b, ValueRef):
                pick = next(((m, o) for m, o in ((a, b), (b, a))
                             if defs.get(m.id) is not None and defs[m.id].op == "mul"), None)
                if pick is not None:
                    mul_inst = defs[pick[0].id]
                    x, y = mul_inst.args
                    if (isinstance(x, ValueRef) and isinstance(y, ValueRef)
                            and inst.out.dtype == DType.F32 and mul_inst.out.dtype == DType.F32
                            and uses.get(mul_inst.out.id, 0) == 1):
                        fused_muls.add(mul_inst.out.id)
                        out.append(Inst("fma", inst.out, (x, y, pick[1])))
                        continue
        out.append(inst)
    kept = tuple(i for i in out if not (i.op == "mul" and i.out is not None and i.out.id in fused_muls))
    return IRModule(ir.name, ir.args, kept)


def _fold_static_lts(ir: IRModule) -> IRModule:
    """Fold ``lt`` to a bool constant when integer intervals decide it.

    Intervals come from constants, ``arange``/``tid`` ranges and ``thread_id``
    (taken as ``[0, NT-1]`` exactly as the reference does), propagated through
    ``add`` and ``mul`` (reference ``compiler.py:658-795``).
    """
    defs = _defs(ir)
    nt = _single_tid_size(ir)
    itv: dict[int, tuple[int, int]] = {}

    def const_int(ref: ValueRef) -> int | None:
        d = defs.get(ref.id)
        if d is None or d.op != "const" or isinstance(d.args[0], bool) or not isinstance(d.args[0], int):
            return None
        return int(d.args[0])

    for inst in ir.insts:
        o = inst.out
        if o is None:
            continue
        if inst.op == "const":
            v = inst.args[0]
            if isinstance(v, int) and not isinstance(v, bool):
                itv[o.id] = (v, v)
        elif inst.op in ("arange", "tid"):
            s, n = int(inst.args[0]), int(inst.args[1])
            itv[o.id] = (s, s + n - 1)
        elif inst.op == "thread_id" and nt is not None:
            itv[o.id] = (0, nt - 1)
        elif inst.op in ("add", "mul"):
            a, b = inst.args
            if not (isinstance(a, ValueRef) and isinstance(b, ValueRef)):
                continue
            ia, ib = itv.get(a.id), itv.get(b.id)
            if inst.op == "add":
                if ia is not None and ib is not None:
                    itv[o.id] = (ia[0] + ib[0], ia[1] + ib[1])
                continue
            if ia is not None and ib is not None:
                corners = [ia[0] * ib[0], ia[0] * ib[1], ia[1] * ib[0], ia[1] * ib[1]]
            elif const_int(a) is not None and ib is not None:
                corners = [const_int(a) * ib[0], const_int(a) * ib[1]]  # type: ignore[operator]
            elif const_int(b) is not None and ia is not None:
                corners = [const_int(b) * ia[0], const_int(b) * ia[1]]  # type: ignore[operator]
            else:
                continue
            itv[o.id] = (min(corners), max(corners))

    table: dict[int, ValueRef] = {}
    remap = _remapper(table)
    out: list[Inst] = []
    for inst in ir.insts:
        args = remap(inst.args)
        o = inst.out
        if o is None:
            out.append(Inst(inst.op, None, args))
            continue
        if inst.op == "lt" and o.dtype == DType.BOOL:
            a, b = args
            if isinstance(a, ValueRef) and isinstance(b, ValueRef):
                ia, ib = itv.get(a.id), itv.get(b.id)
                if ia is not None and ib is not None:
                    decided = True if ia[1] < ib[0] else (False if ia[0] >= ib[1] else None)
                    if decided is not None:
                        out.append(Inst("const", o, (decided,)))
                        table[o.id] = o
                        continue
        out.append(Inst(inst.op, o, args))
        table[o.id] = o
    return IRModule(ir.name, ir.args, tuple(out))


def _simplify_bools(ir: IRModule) -> IRModule:
    """Constant-fold and/or/not and bool-valued ``where`` (reference ``compiler.py:798-934``).

    Constness is judged on the instructions as they were before this pass.
    """
    original = _defs(ir)

    def cbool(ref: ValueRef) -> bool | None:
        d = original.get(ref.id)
        if d is None or d.op != "const" or ref.dtype != DType.BOOL or not isinstance(d.args[0], bool):
            return None
        return bool(d.args[0])

    table: dict[int, ValueRef] = {}
    remap = _remapper(table)
    out: list[Inst] = []

    def keep(op: str, o: ValueRef, args: tuple[Any, ...]) -> None:
        out.append(Inst(op, o, args))  # type: ignore[arg-type]
        table[o.id] = o

    for inst in ir.insts:
        args = remap(inst.args)
        o = inst.out
        if inst.op == "arg" or inst.op in SIDE_EFFECT_OPS or o is None:
            out.append(Inst(inst.op, o, args))
            if o is not None:
                table[o.id] = o
            continue
        if inst.op == "where" and o.dtype == DType.BOOL:
            c, a, b = args
            cc, ca, cb = cbool(c), cbool(a), cbool(b)
            if cc is not None:
                table[o.id] = a if cc else b
                continue
            if cb is False:
                if ca is True:
                    table[o.id] = c
                else:
                    keep("and", o, (c, a))
                continue
            if ca is True and cb is not None:
                keep("or", o, (c, b))
                continue
            if ca is False and cb is not None:
                keep("where", o, (c, a, b))
                continue
        elif inst.op in ("and", "or"):
            a, b = args
            ca, cb = cbool(a), cbool(b)
            absorbing = inst.op == "or"  # value that decides the result on its own
            if ca is absorbing or cb is absorbing:
                keep("const", o, (absorbing,))
                continue
            if ca is (not absorbing):
                table[o.id] = b
                continue
            if cb is (not absorbing):
                table[o.id] = a
                continue
        elif inst.op == "not":
            cx = cbool(args[0])
            if cx is not None:
                keep("const", o, (not cx,))
                continue
        keep(inst.op, o, args)
    return IRModule(ir.name, ir.args, tuple(out))


def _cse_key(inst: Inst, o: ValueRef) -> tuple[Any, ...] | None:
    op, args = inst.op, inst.args
    if op == "const":
        return (op, o.dtype, o.lanes, args[0])
    if op in ("program_id", "thread_id", "local_id"):
        return (op, o.dtype, o.lanes, int(args[0]))
    if op in ("lane_id", "sg_id"):
        return (op, o.dtype, o.lanes)
    if op in ("arange", "tid"):
        return (op, o.dtype, o.lanes, int(args[0]), int(args[1]))
    if op in ("add", "mul", "and", "or"):
        x, y = sorted((args[0].id, args[1].id))
        return (op, o.dtype, o.lanes, x, y)
    if op in ("floordiv", "mod", "lt"):
        return (op, o.dtype, o.lanes, args[0].id, args[1].id)
    if op == "not":
        return (op, o.dtype, o.lanes, args[0].id)
    if op == "where":
        return (op, o.dtype, o.lanes, args[0].id, args[1].id, args[2].id)
    if op == "cast":
        return (op, o.dtype, o.lanes, args[0].id, args[1])
    if op == "fma":
        x, y = sorted((args[0].id, args[1].id))
        return (op, o.dtype, o.lanes, x, y, args[2].id)
    return None


def _cse_pure(ir: IRModule) -> IRModule:
    """Value-number pure ops (commutative operands sorted by id) (reference ``compiler.py:1099-1200``)."""
    table: dict[int, ValueRef] = {}
    remap = _remapper(table)
    numbering: dict[tuple[Any, ...], ValueRef] = {}
    out: list[Inst] = []
    for inst in ir.insts:
        args = remap(inst.args)
        o = inst.out
        if inst.op == "arg" or inst.op in SIDE_EFFECT_OPS or o is None:
            out.append(Inst(inst.op, o, args))
            if o is not None:
                table[o.id] = o
            continue
        key = _cse_key(Inst(inst.op, o, args), o)
        if key is not None and key in numbering:
            table[o.id] = numbering[key]
            continue
        if key is not None:
            numbering[key] = o
        table[o.id] = o
        out.append(Inst(inst.op, o, args))
    return IRModule(ir.name, ir.args, tuple(out))


def _dce(ir: IRModule) -> IRModule:
    """Drop values that no store / mma_store needs; args, arange, tid and barriers stay."""
    defs = _defs(ir)
    live: set[int] = set()
    work: list[int] = []

    def mark(ref: Any) -> None:
        if isinstance(ref, ValueRef) and ref.id not in live:
            live.add(ref.id)
            work.append(ref.id)

    for inst in ir.insts:
        if inst.op in ("store", "mma_store"):
            for a in inst.args:
                mark(a)
        elif inst.op in ("arange", "tid", "arg"):
            mark(inst.out)
    while work:
        d = defs.get(work.pop())
        if d is not None:
            for a in d.args:
                mark(a)
    kept = tuple(i for i in ir.insts
                 if i.op in ("arg", "store", "arange", "tid", "barrier") or i.out is None or i.out.id in live)
    return IRModule(ir.name, ir.args, kept)


def compile_ir(ir: IRModule, *, optimize: bool = False) -> CompiledKernel:
    """Lower an already-traced ``IRModule`` (e.g. one built by hand or loaded from disk)."""
    if optimize:
        ir = optimize_ir(ir)
    validate_ir(ir)
    from .codegen.cuda import ir_to_cuda

    lowered = ir_to_cuda(ir)
    return CompiledKernel(ir=ir, src=lowered.src, block_size=lowered.block_size, launch_mode=lowered.mode,
                          writes=infer_writes(ir), plan=lowered)
