"""SSA intermediate representation produced by the tracer.

The data model (``DType``, ``ValueRef``, ``Arg``, ``Inst``, ``IRModule``) keeps
the field names, dtype strings and op names of the reference IR
(easy_as ``eas/ir.py:10-75``) because user tests build ``IRModule`` objects by
hand and the CUDA emitter, the CPU oracle and the golden fixtures all speak
this format.  The validator is table driven: each op has one checker function
that states the typing rule of the reference validator (``eas/ir.py:86-518``).
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Any, Callable, Iterable, Literal, TypeAlias


class DType(str, Enum):
    BOOL = "bool"
    F16 = "f16"
    F32 = "f32"
    U32 = "u32"
    SG_F32_8X8 = "sg_f32_8x8"


ArgKind: TypeAlias = Literal["buffer", "scalar"]

Op: TypeAlias = Literal[
    "arg", "const", "program_id", "thread_id", "local_id", "lane_id", "sg_id",
    "arange", "tid", "alloc_tg", "add", "mul", "floordiv", "mod", "lt", "and",
    "or", "not", "where", "cast", "dot", "mma_zero", "mma", "mma_store", "load",
    "store", "fma", "barrier",
]

ALL_OPS: frozenset[str] = frozenset(Op.__args__)  # type: ignore[attr-defined]

#: ops that touch memory or synchronise; passes never reorder, merge or drop them
SIDE_EFFECT_OPS = frozenset({"store", "load", "dot", "mma", "mma_store", "alloc_tg", "barrier"})


@dataclass(frozen=True, slots=True)
class ValueRef:
    id: int
    dtype: DType
    lanes: int = 1


@dataclass(frozen=True, slots=True)
class Arg:
    name: str
    dtype: DType
    kind: ArgKind


@dataclass(frozen=True, slots=True)
class Inst:
    op: Op
    out: ValueRef | None
    args: tuple[Any, ...]


@dataclass(frozen=True, slots=True)
class IRModule:
    name: str
    args: tuple[Arg, ...]
    insts: tuple[Inst, ...]

    def buffer_args(self) -> Iterable[Arg]:
        return (a for a in self.args if a.kind == "buffer")

    def scalar_args(self) -> Iterable[Arg]:
        return (a for a in self.args if a.kind == "scalar")


# --------------------------------------------------------------------------
# validation
# --------------------------------------------------------------------------

_NUMERIC = (DType.U32, DType.F16, DType.F32)
_FLOAT = (DType.F16, DType.F32)
_CASTABLE = (DType.BOOL, DType.U32, DType.F16, DType.F32)


class _Checker:
    def __init__(self, ir: IRModule) -> None:
        self.ir = ir
        self.arg_by_name = {a.name: a for a in ir.args}
        self.seen_args: set[str] = set()
        self.defined: dict[int, ValueRef] = {}
        self.buffers: set[int] = set()

    # -- helpers -----------------------------------------------------------
    @staticmethod
    def need(cond: bool, msg: str) -> None:
        if not cond:
            raise ValueError(f"invalid IR: {msg}")

    def define(self, ref: ValueRef | None, what: str) -> ValueRef:
        self.need(ref is not None, f"{what} must produce a value")
        assert ref is not None
        self.need(ref.id not in self.defined, f"duplicate SSA value id: {ref.id}")
        self.need(isinstance(ref.dtype, DType), f"invalid dtype for v{ref.id}: {ref.dtype!r}")
        self.need(isinstance(ref.lanes, int) and ref.lanes >= 1, f"invalid lanes for v{ref.id}: {ref.lanes!r}")
        self.defined[ref.id] = ref
        return ref

    def use(self, x: Any, what: str) -> ValueRef:
        self.need(isinstance(x, ValueRef), f"{what} must be a ValueRef, got {type(x)!r}")
        self.need(x.id in self.defined, f"use of undefined value id {x.id} for {what}")
        d = self.defined[x.id]
        self.need(d.dtype == x.dtype, f"{what} dtype mismatch for v{x.id}: {d.dtype} vs {x.dtype}")
        self.need(d.lanes == x.lanes, f"{what} lanes mismatch for v{x.id}: {d.lanes} vs {x.lanes}")
        return x

    def nargs(self, inst: Inst, n: int) -> None:
        self.need(len(inst.args) == n, f"{inst.op} expects {n} args, got {len(inst.args)}")

    def bcast(self, a: int, b: int, what: str) -> int:
        if a == b or b == 1:
            return a
        if a == 1:
            return b
        raise ValueError(f"invalid IR: {what} lanes mismatch: {a} vs {b} (no broadcast)")

    def buffer(self, x: Any, what: str) -> ValueRef:
        ref = self.use(x, what)
        self.need(ref.id in self.buffers, f"{what} must be a buffer (arg or alloc_tg)")
        return ref

    def scalar_u32(self, x: Any, what: str) -> ValueRef:
        ref = self.use(x, what)
        self.need(ref.dtype == DType.U32, f"{what} must be u32")
        self.need(ref.lanes == 1, f"{what} must be scalar (lanes=1)")
        return ref

    # -- per-op rules ------------------------------------------------------
    def op_arg(self, inst: Inst) -> None:
        self.nargs(inst, 3)
        name, kind, dtype = str(inst.args[0]), inst.args[1], inst.args[2]
        self.need(name in self.arg_by_name, f"arg references unknown name {name!r}")
        decl = self.arg_by_name[name]
        self.need(kind == decl.kind, f"arg kind mismatch for {name!r}")
        self.need(dtype == decl.dtype, f"arg dtype mismatch for {name!r}")
        self.need(name not in self.seen_args, f"duplicate arg inst for {name!r}")
        self.seen_args.add(name)
        out = self.define(inst.out, "arg")
        if decl.kind == "buffer":
            self.buffers.add(out.id)

    def op_const(self, inst: Inst) -> None:
        self.nargs(inst, 1)
        out = inst.out
        self.need(out is not None and out.lanes == 1, "const output lanes must be 1")
        assert out is not None
        v = inst.args[0]
        if out.dtype == DType.BOOL:
            self.need(isinstance(v, bool), "bool const must be a Python bool")
        elif out.dtype == DType.U32:
            self.need(isinstance(v, int) and not isinstance(v, bool) and v >= 0,
                      "u32 const must be a non-negative Python int")
        elif out.dtype == DType.F32:
            self.need(isinstance(v, (int, float)), "f32 const must be an int/float")
        else:
            self.need(False, f"unsupported const dtype: {out.dtype}")
        self.define(out, "const")

    def op_alloc_tg(self, inst: Inst) -> None:
        self.nargs(inst, 1)
        out = self.define(inst.out, "alloc_tg")
        self.need(out.lanes == 1, "alloc_tg output lanes must be 1")
        size = inst.args[0]
        self.need(isinstance(size, int) and size > 0, "alloc_tg(size) requires a positive Python int size")
        self.need(out.dtype in _FLOAT, f"alloc_tg output must be f16/f32, got {out.dtype}")
        self.buffers.add(out.id)

    def op_axis_id(self, inst: Inst) -> None:
        self.nargs(inst, 1)
        out = self.define(inst.out, inst.op)
        self.need(out.lanes == 1 and out.dtype == DType.U32, f"{inst.op} output must be scalar u32")
        self.need(isinstance(inst.args[0], int) and inst.args[0] in (0, 1, 2), f"{inst.op} axis must be 0/1/2")

    def op_range(self, inst: Inst) -> None:
        self.nargs(inst, 2)
        start, size = inst.args
        self.need(isinstance(start, int) and isinstance(size, int),
                  f"{inst.op}(start, size) requires Python int literals")
        self.need(size > 0, f"{inst.op}(size) must be > 0")
        out = self.define(inst.out, inst.op)
        self.need(out.dtype == DType.U32, f"{inst.op} output must be u32")
        want = size if inst.op == "arange" else 1
        self.need(out.lanes == want, f"{inst.op} output lanes must be {want}")

    def op_lane_sg(self, inst: Inst) -> None:
        self.nargs(inst, 0)
        out = self.define(inst.out, inst.op)
        self.need(out.dtype == DType.U32 and out.lanes == 1, f"{inst.op} output must be scalar u32")

    def op_arith(self, inst: Inst) -> None:
        self.nargs(inst, 2)
        a = self.use(inst.args[0], f"{inst.op} lhs")
        b = self.use(inst.args[1], f"{inst.op} rhs")
        self.need(a.dtype == b.dtype, f"{inst.op} dtype mismatch: {a.dtype} vs {b.dtype}")
        self.need(a.dtype in _NUMERIC, f"{inst.op} operands must be u32/f16/f32, got {a.dtype}")
        if inst.op in ("floordiv", "mod"):
            self.need(a.dtype == DType.U32, f"{inst.op} operands must be u32")
        lanes = self.bcast(a.lanes, b.lanes, f"{inst.op} operands")
        out = inst.out
        self.need(out is not None and out.dtype == a.dtype, f"{inst.op} output dtype must match operands")
        self.need(out.lanes == lanes, f"{inst.op} output lanes must broadcast operands")  # type: ignore[union-attr]
        self.define(out, inst.op)

    def op_lt(self, inst: Inst) -> None:
        self.nargs(inst, 2)
        a = self.use(inst.args[0], "lt lhs")
        b = self.use(inst.args[1], "lt rhs")
        self.need(a.dtype == b.dtype, f"lt dtype mismatch: {a.dtype} vs {b.dtype}")
        self.need(a.dtype in _NUMERIC, "lt operands must be u32/f16/f32")
        out = self.define(inst.out, "lt")
        self.need(out.dtype == DType.BOOL, "lt output must be bool")
        self.need(out.lanes == self.bcast(a.lanes, b.lanes, "lt operands"), "lt output lanes mismatch")

    def op_logic(self, inst: Inst) -> None:
        self.nargs(inst, 2)
        a = self.use(inst.args[0], f"{inst.op} lhs")
        b = self.use(inst.args[1], f"{inst.op} rhs")
        self.need(a.dtype == DType.BOOL and b.dtype == DType.BOOL, f"{inst.op} operands must be bool")
        out = self.define(inst.out, inst.op)
        self.need(out.dtype == DType.BOOL, f"{inst.op} output must be bool")
        self.need(out.lanes == self.bcast(a.lanes, b.lanes, inst.op), f"{inst.op} output lanes mismatch")

    def op_not(self, inst: Inst) -> None:
        self.nargs(inst, 1)
        x = self.use(inst.args[0], "not input")
        out = self.define(inst.out, "not")
        self.need(x.dtype == DType.BOOL and out.dtype == DType.BOOL, "not operates on bool")
        self.need(out.lanes == x.lanes, "not output lanes must match input")

    def op_where(self, inst: Inst) -> None:
        self.nargs(inst, 3)
        c = self.use(inst.args[0], "where cond")
        a = self.use(inst.args[1], "where a")
        b = self.use(inst.args[2], "where b")
        self.need(c.dtype == DType.BOOL, "where cond must be bool")
        self.need(a.dtype == b.dtype, f"where dtype mismatch: {a.dtype} vs {b.dtype}")
        out = self.define(inst.out, "where")
        self.need(out.dtype == a.dtype, "where output dtype must match values")
        lanes = self.bcast(c.lanes, self.bcast(a.lanes, b.lanes, "where values"), "where cond vs values")
        self.need(out.lanes == lanes, "where output lanes mismatch")

    def op_cast(self, inst: Inst) -> None:
        self.nargs(inst, 2)
        x = self.use(inst.args[0], "cast input")
        dst = inst.args[1]
        self.need(isinstance(dst, DType), "cast target must be a DType")
        out = self.define(inst.out, "cast")
        self.need(out.dtype == dst, "cast output dtype must match target dtype")
        self.need(out.lanes == x.lanes, "cast output lanes must match input")
        self.need(x.dtype in _CASTABLE and dst in _CASTABLE, "cast only supports bool/u32/f16/f32")

    def op_load(self, inst: Inst) -> None:
        self.nargs(inst, 3)
        buf = self.buffer(inst.args[0], "load buffer")
        off = self.use(inst.args[1], "load offset")
        mask = self.use(inst.args[2], "load mask")
        self.need(buf.dtype in _FLOAT, "load buffer dtype must be f16/f32")
        self.need(off.dtype == DType.U32, "load offset must be u32")
        self.need(mask.dtype == DType.BOOL, "load mask must be bool")
        out = self.define(inst.out, "load")
        self.need(out.dtype == buf.dtype, "load output dtype must match buffer dtype")
        self.need(out.lanes == off.lanes, "load output lanes must match offset lanes")
        self.need(mask.lanes in (1, off.lanes), "load mask lanes must be 1 or match offset lanes")

    def op_store(self, inst: Inst) -> None:
        self.nargs(inst, 4)
        self.need(inst.out is None, "store must not produce a value")
        buf = self.buffer(inst.args[0], "store buffer")
        off = self.use(inst.args[1], "store offset")
        val = self.use(inst.args[2], "store value")
        mask = self.use(inst.args[3], "store mask")
        self.need(buf.dtype in _FLOAT, "store buffer dtype must be f16/f32")
        self.need(off.dtype == DType.U32, "store offset must be u32")
        self.need(mask.dtype == DType.BOOL, "store mask must be bool")
        self.need(val.dtype == buf.dtype, "store value dtype must match buffer dtype")
        self.need(val.lanes in (1, off.lanes), "store value lanes must be 1 or match offset lanes")
        self.need(mask.lanes in (1, off.lanes), "store mask lanes must be 1 or match offset lanes")

    def op_fma(self, inst: Inst) -> None:
        self.nargs(inst, 3)
        x = self.use(inst.args[0], "fma x")
        y = self.use(inst.args[1], "fma y")
        z = self.use(inst.args[2], "fma z")
        self.need(x.dtype == y.dtype == z.dtype, "fma operands must have same dtype")
        self.need(x.dtype in _FLOAT, "fma operands must be f16/f32")
        out = self.define(inst.out, "fma")
        self.need(out.dtype == x.dtype, "fma output dtype must match operands")
        lanes = self.bcast(z.lanes, self.bcast(x.lanes, y.lanes, "fma x/y"), "fma z vs x/y")
        self.need(out.lanes == lanes, "fma output lanes mismatch")

    def _matrix_operands(self, inst: Inst, what: str) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride = inst.args[:6]
        for ref, nm in ((a_buf, "a_buffer"), (b_buf, "b_buffer")):
            r = self.buffer(ref, f"{what} {nm}")
            self.need(r.dtype in _FLOAT, f"{what} {nm} must be f16/f32")
        for ref, nm in ((a_base, "a_base"), (a_stride, "a_stride"), (b_base, "b_base"), (b_stride, "b_stride")):
            self.scalar_u32(ref, f"{what} {nm}")

    def op_dot(self, inst: Inst) -> None:
        self.nargs(inst, 7)
        self._matrix_operands(inst, "dot")
        self.scalar_u32(inst.args[6], "dot K")
        out = self.define(inst.out, "dot")
        self.need(out.lanes == 1 and out.dtype == DType.F32, "dot output must be scalar f32")

    def op_mma_zero(self, inst: Inst) -> None:
        self.nargs(inst, 0)
        out = self.define(inst.out, "mma_zero")
        self.need(out.dtype == DType.SG_F32_8X8 and out.lanes == 1, "mma_zero produces sg_f32_8x8")

    def op_mma(self, inst: Inst) -> None:
        self.nargs(inst, 7)
        self._matrix_operands(inst, "mma")
        acc = self.use(inst.args[6], "mma acc")
        self.need(acc.dtype == DType.SG_F32_8X8 and acc.lanes == 1, "mma acc must be sg_f32_8x8")
        out = self.define(inst.out, "mma")
        self.need(out.dtype == DType.SG_F32_8X8 and out.lanes == 1, "mma produces sg_f32_8x8")

    def op_mma_store(self, inst: Inst) -> None:
        self.nargs(inst, 4)
        self.need(inst.out is None, "mma_store must not produce a value")
        buf = self.buffer(inst.args[0], "mma_store c_buffer")
        self.need(buf.dtype == DType.F32, "mma_store c_buffer must be f32")
        self.scalar_u32(inst.args[1], "mma_store c_base")
        self.scalar_u32(inst.args[2], "mma_store c_stride")
        frag = self.use(inst.args[3], "mma_store frag")
        self.need(frag.dtype == DType.SG_F32_8X8 and frag.lanes == 1, "mma_store frag must be sg_f32_8x8")

    def op_barrier(self, inst: Inst) -> None:
        self.nargs(inst, 0)
        self.need(inst.out is None, "barrier must not produce a value")

    RULES: dict[str, Callable[["_Checker", Inst], None]] = {}

    def run(self) -> None:
        for inst in self.ir.insts:
            self.need(inst.op in ALL_OPS, f"unknown op: {inst.op!r}")
            self.RULES[inst.op](self, inst)
        missing = set(self.arg_by_name) - self.seen_args
        self.need(not missing, "missing arg inst(s): " + ", ".join(sorted(missing)))


_Checker.RULES = {
    "arg": _Checker.op_arg, "const": _Checker.op_const, "alloc_tg": _Checker.op_alloc_tg,
    "program_id": _Checker.op_axis_id, "thread_id": _Checker.op_axis_id, "local_id": _Checker.op_axis_id,
    "arange": _Checker.op_range, "tid": _Checker.op_range,
    "lane_id": _Checker.op_lane_sg, "sg_id": _Checker.op_lane_sg,
    "add": _Checker.op_arith, "mul": _Checker.op_arith, "floordiv": _Checker.op_arith, "mod": _Checker.op_arith,
    "lt": _Checker.op_lt, "and": _Checker.op_logic, "or": _Checker.op_logic, "not": _Checker.op_not,
    "where": _Checker.op_where, "cast": _Checker.op_cast, "load": _Checker.op_load, "store": _Checker.op_store,
    "fma": _Checker.op_fma, "dot": _Checker.op_dot, "mma_zero": _Checker.op_mma_zero, "mma": _Checker.op_mma,
    "mma_store": _Checker.op_mma_store, "barrier": _Checker.op_barrier,
}


def validate_ir(ir: IRModule) -> None:
    """Raise ``ValueError("invalid IR: ...")`` if ``ir`` breaks a typing rule."""
    _Checker(ir).run()


# --------------------------------------------------------------------------
# JSON form (the fixture format of tests/golden: plain lists, value refs as {"v": [id, dtype, lanes]})
# --------------------------------------------------------------------------

def _arg_from_json(x: Any) -> Any:
    if isinstance(x, dict) and "v" in x:
        i, dt, lanes = x["v"]
        return ValueRef(int(i), DType(dt), int(lanes))
    if isinstance(x, dict) and "dt" in x:
        return DType(x["dt"])
    return x


def ir_from_json(d: dict) -> IRModule:
    args = tuple(Arg(n, DType(dt), kind) for n, dt, kind in d["args"])
    insts = []
    for op, out, a in d["insts"]:
        o = None if out is None else ValueRef(int(out[0]), DType(out[1]), int(out[2]))
        insts.append(Inst(op, o, tuple(_arg_from_json(x) for x in a)))
    return IRModule(d["name"], args, tuple(insts))


def ir_to_json(ir: IRModule) -> dict:
    def ser(a: Any) -> Any:
        if isinstance(a, ValueRef):
            return {"v": [a.id, a.dtype.value, a.lanes]}
        if isinstance(a, DType):
            return {"dt": a.value}
        return a

    return {"name": ir.name, "args": [[a.name, a.dtype.value, a.kind] for a in ir.args],
            "insts": [[i.op, None if i.out is None else [i.out.id, i.out.dtype.value, i.out.lanes],
                       [ser(x) for x in i.args]] for i in ir.insts]}
