"""Lower traced IR to CUDA C++ for sm_100a (compiled at run time by NVRTC).

This replaces the reference's Metal emitter (easy_as ``eas/codegen/msl.py``)
and keeps its execution semantics, re-mapped onto the CUDA machine:

Mode inference (``msl.py:59-95``)
    ``mk.arange(0, BLOCK)`` makes an SPMD kernel, ``mk.tid(0, BLOCK)`` a
    thread kernel; the two never mix and only one size is allowed.

SPMD kernels (Metal: one thread walks a ``BLOCK``-lane array, ``msl.py:98-350``)
    One *program* is one CTA.  Its ``BLOCK`` lanes are spread over ``T``
    threads, ``V`` consecutive lanes per thread per chunk, chunks ``T*V``
    lanes apart, so a warp touches 32*V consecutive elements per chunk.
    A load or store whose offset is ``scalar + arange`` (unit lane stride)
    becomes one 16-byte vector access per chunk when the address is aligned
    and all ``V`` lane masks are set, else per-lane predicated accesses.
    Scalar (lane-uniform) stores are done by thread 0 only, and a
    ``__syncthreads()`` follows any store that later memory operations could
    observe, so the program still behaves as one sequential instruction
    stream.

Thread kernels (one Metal thread per ``tid``, ``msl.py:353-1433``)
    One CUDA thread per DSL thread, ``blockDim.x = BLOCK``.  A 1D launch
    without ``_grid`` runs exactly ``N`` threads in Metal (partial last group,
    ``metal.py:283-288``): threads past ``N`` return at once when the kernel
    has no barriers, block memory or matrix ops, and otherwise stay alive as
    inert "ghosts" that join barriers and warp matrix ops but never touch
    memory.

Operations
    ``mul``/``add`` stay separately rounded (NVRTC ``--fmad=false``); ``fma``
    is ``fmaf``; f16 values are carried as their bit pattern and computed in
    f32 with one round-to-nearest-even at the end (exactly rounded for
    ``+``/``*``, as in ``msl.py:885-897`` for ``fma``); ``dot`` is the strict
    ``k``-order ``fmaf`` chain from 0 (``msl.py:920-952``); ``mma`` is one
    warp-wide ``mma.sync.m16n8k8`` (f16 operands, f32 accumulate) holding the
    8x8 fragment in rows 0-7, or an FFMA loop for f32 operands.

Hidden parameters follow the IR arguments: ``eas_ntx`` (active threads along
x, thread mode) and ``eas_pid_{x,y,z}`` (program-id offsets, used to split a
grid into several launches or across GPUs).

Bounds-checked mode (``EAS_BOUNDS_CHECK=1``, read when a specialisation is
compiled): every buffer gets two more hidden parameters, ``eas_lo_<name>`` and
``eas_n_<name>`` (u64: the buffer holds global elements [lo, lo + n)), and the
kernel takes ``eas_err``, a pointer to four u32 words.  Every global and
threadgroup access whose mask holds is first tested against its buffer; an
access outside is skipped (a load yields 0) and the first one is recorded as
(1, 2 * slot + is_store, index, 0), slot being the buffer's position in the
argument list or ``CHECK_TG_SLOT`` + the threadgroup allocation's order.  The
runtime clears the record before the launch and raises after it.  Vector
accesses and grouped dot loops are off in this mode, so each element is
tested on its own.
"""

from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from ..ir import DType, IRModule, Inst, ValueRef
from .reroll import Run, find_runs

# ---------------------------------------------------------------------------
# launch description shared with the runtime
# ---------------------------------------------------------------------------


@dataclass(frozen=True, slots=True)
class Param:
    name: str          # C identifier in the kernel signature
    kind: str          # "buffer" | "scalar" | "hidden"
    dtype: DType | None
    arg: str | None    # IR argument name (None for hidden params)


@dataclass(slots=True)
class Lowered:
    src: str
    kernel_name: str
    block_size: int      # DSL BLOCK (spmd lanes per program / thread-mode threads per block)
    mode: str            # "spmd" | "thread"
    cuda_threads: int    # CUDA threads per CTA
    params: list[Param]
    dyn_smem: int        # bytes of dynamic shared memory per CTA
    native: Any = field(default=None)   # pattern-lowered native plan (see codegen.patterns)
    elementwise: Any = field(default=None)  # ElementwiseInfo when program p touches only elements [p*B, p*B+B)
    layout: Any = field(default=None)   # runtime parameter layout, built on first launch
    grid_rank: Any = field(default=None)  # 1 + highest program_id/thread_id axis, cached by the runtime
    reads: frozenset = field(default=frozenset())  # buffer args the kernel may read (analysis.infer_reads)
    checked: bool = False  # bounds-checked lowering (extra "check" params; see the module docstring)


HIDDEN = ("eas_ntx", "eas_pid_x", "eas_pid_y", "eas_pid_z")
CHECK_TG_SLOT = 1000   # error-record slot of the first threadgroup allocation (bounds-checked mode)


def bounds_check_enabled() -> bool:
    """EAS_BOUNDS_CHECK=1: lower kernels with per-access bounds checks (read at compile time)."""
    return os.environ.get("EAS_BOUNDS_CHECK", "0") not in ("", "0", "off", "false")

_CXX_RESERVED = {
    "auto", "bool", "break", "case", "char", "class", "const", "continue", "default", "delete", "do",
    "double", "else", "enum", "extern", "float", "for", "goto", "if", "inline", "int", "long", "new",
    "operator", "private", "protected", "public", "register", "return", "short", "signed", "sizeof",
    "static", "struct", "switch", "template", "this", "throw", "try", "typedef", "union", "unsigned",
    "virtual", "void", "volatile", "while", "half", "dim3", "uint", "asm", "namespace", "using",
    "threadIdx", "blockIdx", "blockDim", "gridDim", "warpSize", "true", "false", "nullptr",
    # the remaining C++ keywords a Python identifier can spell
    "alignas", "alignof", "char16_t", "char32_t", "char8_t", "compl", "bitand", "bitor", "const_cast",
    "constexpr", "consteval", "constinit", "decltype", "dynamic_cast", "explicit", "export", "friend",
    "mutable", "noexcept", "not_eq", "and_eq", "or_eq", "xor", "xor_eq", "reinterpret_cast", "static_assert",
    "static_cast", "thread_local", "typeid", "typename", "wchar_t", "concept", "requires", "co_await",
    "co_return", "co_yield",
    # types and functions the generated code names
    "uint32_t", "uint64_t", "float2", "float4", "make_float2", "fmaf", "atomicCAS",
}


def c_ident(name: str) -> str:
    if name in _CXX_RESERVED or name.startswith("eas_") or name.startswith("__") or (
            name[:1] == "v" and name[1:].isdigit()):
        return f"{name}_p"
    return name


_CTYPE = {DType.F32: "float", DType.F16: "eas_h", DType.U32: "uint32_t", DType.BOOL: "bool",
          DType.SG_F32_8X8: "float2"}


def ctype(dt: DType) -> str:
    return _CTYPE[dt]


def f32_literal(v: float) -> str:
    bits = struct.unpack("<I", struct.pack("<f", float(np.float32(v))))[0]
    return f"__int_as_float(0x{bits:08x})"


def infer_block_and_mode(ir: IRModule) -> tuple[int, str]:
    sizes = {"arange": set(), "tid": set()}
    for inst in ir.insts:
        if inst.op in sizes:
            sizes[inst.op].add(int(inst.args[1]))
    for op, s in sizes.items():
        if len(s) > 1:
            raise ValueError(f"multiple {op} sizes not supported in MVP")
    if sizes["arange"] and sizes["tid"]:
        raise ValueError("kernel must not mix mk.arange(...) and mk.tid(...) in MVP")
    if sizes["arange"]:
        return next(iter(sizes["arange"])), "spmd"
    if sizes["tid"]:
        return next(iter(sizes["tid"])), "thread"
    raise ValueError("kernel must use mk.arange(0, BLOCK) (spmd) or mk.tid(0, BLOCK) (thread) to define BLOCK")


PRELUDE = r"""
typedef unsigned int uint32_t;
typedef unsigned long long uint64_t;
typedef unsigned short eas_h;
struct __align__(8) eas_h4 { eas_h x, y, z, w; };
static __device__ __forceinline__ float eas_h2f(eas_h h) { float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
static __device__ __forceinline__ eas_h eas_f2h(float f) { eas_h h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
static __device__ __forceinline__ eas_h eas_u2h(uint32_t u) { eas_h h; asm("cvt.rn.f16.u32 %0, %1;" : "=h"(h) : "r"(u)); return h; }
static __device__ __forceinline__ uint32_t eas_h2u(eas_h h) { uint32_t u; asm("cvt.rzi.sat.u32.f16 %0, %1;" : "=r"(u) : "h"(h)); return u; }
static __device__ __forceinline__ uint32_t eas_f2u(float f) { uint32_t u; asm("cvt.rzi.sat.u32.f32 %0, %1;" : "=r"(u) : "f"(f)); return u; }
static __device__ __forceinline__ float eas_u2f(uint32_t u) { float f; asm("cvt.rn.f32.u32 %0, %1;" : "=f"(f) : "r"(u)); return f; }
static __device__ __forceinline__ uint32_t eas_pack2(eas_h lo, eas_h hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }
static __device__ __forceinline__ float2 eas_mma_f16(uint32_t a01, uint32_t b01, float2 c) {
  float d0, d1, d2, d3;
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
               : "=f"(d0), "=f"(d1), "=f"(d2), "=f"(d3)
               : "r"(a01), "r"(0u), "r"(b01), "f"(c.x), "f"(c.y), "f"(0.0f), "f"(0.0f));
  return make_float2(d0, d1);
}
"""

CHECK_PRELUDE = r"""
// bounds-checked mode: true when global element i of a buffer holding [lo, lo + n) exists;
// otherwise the first failing access in the launch is recorded in err[0..2]
static __device__ __noinline__ bool eas_inb(uint32_t i, uint64_t lo, uint64_t n, uint32_t* err, uint32_t what) {
  if ((uint64_t)i - lo < n) return true;
  if (atomicCAS(err, 0u, 1u) == 0u) { err[1] = what; err[2] = i; }
  return false;
}
"""

# ---------------------------------------------------------------------------
# helpers for value expressions
# ---------------------------------------------------------------------------


def _zero(dt: DType) -> str:
    return {DType.F32: "0.0f", DType.F16: "(eas_h)0", DType.U32: "0u", DType.BOOL: "false"}[dt]


def _cast_expr(x: str, src: DType, dst: DType) -> str:
    if src == dst:
        return x
    if dst == DType.BOOL:
        return {DType.U32: f"({x} != 0u)", DType.F32: f"({x} != 0.0f)", DType.F16: f"(eas_h2f({x}) != 0.0f)"}[src]
    if src == DType.BOOL:
        return {DType.U32: f"({x} ? 1u : 0u)", DType.F32: f"({x} ? 1.0f : 0.0f)",
                DType.F16: f"({x} ? (eas_h)0x3c00 : (eas_h)0)"}[dst]
    table = {
        (DType.U32, DType.F32): f"eas_u2f({x})",
        (DType.U32, DType.F16): f"eas_u2h({x})",
        (DType.F32, DType.U32): f"eas_f2u({x})",
        (DType.F32, DType.F16): f"eas_f2h({x})",
        (DType.F16, DType.F32): f"eas_h2f({x})",
        (DType.F16, DType.U32): f"eas_h2u({x})",
    }
    return table[(src, dst)]


def _binop_expr(op: str, dt: DType, a: str, b: str, nonzero_b: bool = False) -> str:
    """C expression of a binary IR op.  u32 ``x // 0`` is 0xFFFFFFFF and ``x % 0`` is ``x``
    (the reference leaves these undefined; the oracle uses the same definition)."""
    if op in ("add", "mul"):
        sym = "+" if op == "add" else "*"
        if dt == DType.F16:
            return f"eas_f2h(eas_h2f({a}) {sym} eas_h2f({b}))"
        if dt == DType.F32:
            return f"__f{'add' if op == 'add' else 'mul'}_rn({a}, {b})"
        return f"({a} {sym} {b})"
    if op == "floordiv":
        return f"({a} / {b})" if nonzero_b else f"(({b}) ? ({a} / {b}) : 0xFFFFFFFFu)"
    if op == "mod":
        return f"({a} % {b})" if nonzero_b else f"(({b}) ? ({a} % {b}) : ({a}))"
    if op == "lt":
        if dt == DType.F16:
            return f"(eas_h2f({a}) < eas_h2f({b}))"
        return f"({a} < {b})"
    if op == "and":
        return f"({a} && {b})"
    if op == "or":
        return f"({a} || {b})"
    raise ValueError(op)


def _fma_expr(dt: DType, x: str, y: str, z: str) -> str:
    if dt == DType.F16:
        return f"eas_f2h(fmaf(eas_h2f({x}), eas_h2f({y}), eas_h2f({z})))"
    return f"fmaf({x}, {y}, {z})"


def _as_float(dt: DType, x: str) -> str:
    return f"eas_h2f({x})" if dt == DType.F16 else x


# ---------------------------------------------------------------------------
# emitter
# ---------------------------------------------------------------------------


class _Emitter:
    def __init__(self, ir: IRModule, checked: bool = False):
        self.ir = ir
        self.checked = checked
        # C identifier of each argument: c_ident, made unique ("x" renamed to "x_p" must not meet an
        # argument that is itself called "x_p")
        self.cname: dict[str, str] = {}
        for a in ir.args:
            c = c_ident(a.name)
            while c in self.cname.values():
                c += "_p"
            self.cname[a.name] = c
        self.block, self.mode = infer_block_and_mode(ir)
        self.defs: dict[int, Inst] = {i.out.id: i for i in ir.insts if i.out is not None}
        self.arg_c: dict[int, str] = {}       # value id of an arg -> C identifier
        self.arg_dtype: dict[int, DType] = {}
        self.writes: set[str] = set()
        self.tg: dict[int, tuple[int, int]] = {}   # alloc_tg value id -> (byte offset, elements)
        self.lines: list[str] = []
        self.depth = 0                         # extra indentation (inside re-rolled loops)
        self.alias: dict[int, str] = {}        # value id -> C expression (loop-carried / affine operands)
        self.uses: dict[int, int] = {}
        for inst in ir.insts:
            for a in inst.args:
                if isinstance(a, ValueRef):
                    self.uses[a.id] = self.uses.get(a.id, 0) + 1
        for inst in ir.insts:
            if inst.op == "arg":
                self.arg_c[inst.out.id] = self.cname[str(inst.args[0])]
                self.arg_dtype[inst.out.id] = inst.out.dtype
            elif inst.op in ("store", "mma_store"):
                buf = inst.args[0]
                if buf.id in self.arg_c:
                    self.writes.add(self.arg_c[buf.id])
        self.cooperative = any(i.op in ("barrier", "alloc_tg", "mma_zero", "mma", "mma_store") for i in ir.insts)
        if self.mode == "spmd":
            forbidden = {"tid", "local_id", "lane_id", "sg_id", "dot", "mma_zero", "mma", "mma_store"}
            for inst in ir.insts:
                if inst.op in forbidden:
                    raise ValueError(f"op {inst.op!r} is not supported in spmd mode "
                                     "(use mk.tid for thread-level kernels)")
            self.V = 4 if self.block % 4 == 0 else 1
            per_chunk = self.block // self.V
            self.T = per_chunk if per_chunk <= 256 else 256
            self.J = -(-per_chunk // self.T)
            self.L = self.J * self.V
            self.lane_guard = (self.J * self.T * self.V) != self.block
            self.cuda_threads = self.T
            # unit-stride lane vectors: value id -> C expression of the scalar base
            self.unit: dict[int, str] = {}
        else:
            if self.block > 1024:
                raise ValueError(f"thread mode BLOCK={self.block} exceeds 1024 threads per block")
            self.cuda_threads = self.block
        smem = 0
        for inst in ir.insts:
            if inst.op == "alloc_tg":
                nbytes = int(inst.args[0]) * (4 if inst.out.dtype == DType.F32 else 2)
                self.tg[inst.out.id] = (smem, int(inst.args[0]))
                smem += -(-nbytes // 16) * 16
        self.smem = smem
        # error-record slot of each buffer (bounds-checked mode)
        arg_pos = {a.name: n for n, a in enumerate(ir.args)}
        self.slot: dict[int, int] = {}
        for inst in ir.insts:
            if inst.op == "arg" and str(inst.args[0]) in arg_pos:
                self.slot[inst.out.id] = arg_pos[str(inst.args[0])]
        for n, vid in enumerate(self.tg):
            self.slot[vid] = CHECK_TG_SLOT + n

    # -- naming ---------------------------------------------------------------
    def name(self, ref: ValueRef) -> str:
        a = self.alias.get(ref.id)
        if a is not None:
            return a
        return self.arg_c.get(ref.id, f"v{ref.id}")

    def lane(self, ref: ValueRef, i: str) -> str:
        n = self.name(ref)
        return f"{n}[{i}]" if ref.lanes > 1 else n

    def _nonzero_const(self, ref: ValueRef) -> bool:
        d = self.defs.get(ref.id)
        return d is not None and d.op == "const" and not isinstance(d.args[0], bool) and int(d.args[0]) % (1 << 32) != 0

    def is_const_true(self, ref: ValueRef) -> bool:
        d = self.defs.get(ref.id)
        return d is not None and d.op == "const" and d.args[0] is True and ref.dtype == DType.BOOL

    def inb(self, buf: ValueRef, idx: str, store: bool = False) -> str:
        """Bounds test of one access (checked mode), or "true"."""
        if not self.checked:
            return "true"
        what = 2 * self.slot[buf.id] + int(store)
        if buf.id in self.tg:
            return f"eas_inb({idx}, 0ull, {self.tg[buf.id][1]}ull, eas_err, {what}u)"
        c = self.arg_c[buf.id]
        return f"eas_inb({idx}, eas_lo_{c}, eas_n_{c}, eas_err, {what}u)"

    def ld(self, buf: ValueRef, idx: str) -> str:
        """Read of one element inside a dot or mma: unguarded, or 0 when out of bounds (checked mode)."""
        rhs = f"{self.name(buf)}[{idx}]"
        if not self.checked:
            return rhs
        return f"({self.inb(buf, idx)} ? {rhs} : {_zero(buf.dtype)})"

    @staticmethod
    def both(a: str, b: str) -> str:
        if a == "true":
            return b
        if b == "true":
            return a
        return f"({a} && {b})"

    def emit(self, line: str, indent: int = 1) -> None:
        self.lines.append("  " * (indent + self.depth) + line)

    # -- signature -------------------------------------------------------------
    def params(self) -> list[Param]:
        ps = []
        for a in self.ir.args:
            ps.append(Param(self.cname[a.name], a.kind, a.dtype, a.name))
        ps += [Param(h, "hidden", DType.U32, None) for h in HIDDEN]
        if self.checked:
            for a in self.ir.args:
                if a.kind == "buffer":
                    c = self.cname[a.name]
                    ps += [Param(f"eas_lo_{c}", "check", None, a.name), Param(f"eas_n_{c}", "check", None, a.name)]
            ps.append(Param("eas_err", "check", None, None))
        return ps

    def signature(self) -> str:
        parts = []
        for a in self.ir.args:
            cn = self.cname[a.name]
            if a.kind == "buffer":
                t = ctype(a.dtype)
                if cn in self.writes:
                    parts.append(f"{t}* {cn}")
                else:
                    parts.append(f"const {t}* __restrict__ {cn}")
            else:
                parts.append(f"const {ctype(a.dtype)} {cn}")
        parts += [f"const uint32_t {h}" for h in HIDDEN]
        if self.checked:
            for a in self.ir.args:
                if a.kind == "buffer":
                    c = self.cname[a.name]
                    parts += [f"const uint64_t eas_lo_{c}", f"const uint64_t eas_n_{c}"]
            parts.append("uint32_t* const eas_err")
        return ",\n    ".join(parts)

    # -- main -------------------------------------------------------------------
    def run(self) -> Lowered:
        body = self._spmd() if self.mode == "spmd" else self._thread()
        name = c_ident(self.ir.name) if self.ir.name else "eas_kernel"
        src = "\n".join([
            f"// generated by easy_as_b200.codegen.cuda for sm_100a ({self.mode} mode, BLOCK={self.block})",
            PRELUDE + (CHECK_PRELUDE if self.checked else ""),
            f'extern "C" __global__ void __launch_bounds__({self.cuda_threads}, {self._min_blocks()}) {name}(',
            "    " + self.signature() + ") {",
            # programmatic dependent launch: the next kernel in the stream may be scheduled from now on,
            # and this one touches no memory before the previous grid has completed (both are no-ops
            # for a launch without the attribute)
            '    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");',
            '    asm volatile("griddepcontrol.wait;" ::: "memory");',
            *body,
            "}",
            "",
        ])
        return Lowered(src=src, kernel_name=name, block_size=self.block, mode=self.mode,
                       cuda_threads=self.cuda_threads, params=self.params(), dyn_smem=self.smem,
                       checked=self.checked)

    def _min_blocks(self) -> int:
        """CTAs per SM to plan registers for: enough for 2048 resident threads (<= 64 registers each),
        as far as the block's shared memory allows."""
        want = max(1, 2048 // self.cuda_threads)
        if self.smem:
            want = min(want, max(1, (200 * 1024) // self.smem))
        return min(want, 32)

    def _smem_decls(self) -> None:
        if not self.tg:
            return
        self.emit("extern __shared__ __align__(16) unsigned char eas_smem[];")
        for vid, (off, _n) in self.tg.items():
            dt = self.defs[vid].out.dtype
            self.emit(f"{ctype(dt)}* const v{vid} = reinterpret_cast<{ctype(dt)}*>(eas_smem + {off});")

    # ======================================================================
    # SPMD
    # ======================================================================
    def _lane_index(self, i: int) -> str:
        j, e = divmod(i, self.V)
        return f"({j * self.T * self.V}u + threadIdx.x * {self.V}u + {e}u)"

    def _spmd(self) -> list[str]:
        L = self.L
        self.emit(f"// {self.T} threads x {self.L} lanes each ({self.J} chunk(s) of {self.V})")
        self._smem_decls()
        if self.lane_guard:
            self.emit(f"bool eas_lv[{L}];")
            for i in range(L):
                self.emit(f"eas_lv[{i}] = {self._lane_index(i)} < {self.block}u;")
        insts = self.ir.insts
        mem_after = [False] * len(insts)
        seen = False
        for k in range(len(insts) - 1, -1, -1):
            mem_after[k] = seen
            if insts[k].op in ("load", "store"):
                seen = True
        runs = find_runs(insts) if os.environ.get("EAS_REROLL", "1") != "0" else []
        run_at = {r.first[0]: r for r in runs}
        in_run: set[int] = set()
        for r in runs:
            in_run |= r.ir_span
        if runs:  # constants first: re-rolled blocks read them from any position
            for inst in insts:
                if inst.op == "const":
                    self._spmd_inst(inst)

        def block(run: Run, body: dict[int, Inst]) -> None:
            for k in run.first:
                self._spmd_inst(body[k])
                if body[k].op == "store" and mem_after[k]:
                    self.emit("__syncthreads();")

        for k, inst in enumerate(insts):
            if runs and inst.op == "const":
                continue
            if k in run_at:
                self._emit_run(run_at[k], lambda body, r=run_at[k]: block(r, body))
            if k in in_run:
                continue
            self._spmd_inst(inst)
            if inst.op == "store" and mem_after[k]:
                self.emit("__syncthreads();")
        return self.lines

    def _vec_decl(self, out: ValueRef) -> str:
        return f"{ctype(out.dtype)} v{out.id}[{self.L}];"

    def _spmd_elementwise(self, out: ValueRef, expr_of_i) -> None:
        if out.lanes == 1:
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {expr_of_i('0')};")
            return
        self.emit(self._vec_decl(out))
        self.emit(f"#pragma unroll\nfor (int eas_i = 0; eas_i < {self.L}; ++eas_i) v{out.id}[eas_i] = {expr_of_i('eas_i')};")

    def _spmd_inst(self, inst: Inst) -> None:
        op, out, args = inst.op, inst.out, inst.args
        if op in ("arg", "alloc_tg"):
            return
        if op == "const":
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {self._const(out.dtype, args[0])};")
            return
        if op in ("program_id", "thread_id"):
            ax = "xyz"[int(args[0])]
            self.emit(f"const uint32_t v{out.id} = blockIdx.{ax} + eas_pid_{ax};")
            return
        if op == "arange" and out.lanes == 1:
            self.emit(f"const uint32_t v{out.id} = {int(args[0])}u;")  # BLOCK == 1: one lane, held by thread 0
            return
        if op == "arange":
            start = int(args[0])
            self.emit(self._vec_decl(out))
            for i in range(self.L):
                self.emit(f"v{out.id}[{i}] = {start}u + {self._lane_index(i)};")
            self.unit[out.id] = f"{start}u"
            return
        if op in ("add", "mul", "floordiv", "mod", "lt", "and", "or"):
            a, b = args
            dt = a.dtype
            nz = self._nonzero_const(b)
            self._spmd_elementwise(out, lambda i: _binop_expr(op, dt, self.lane(a, i), self.lane(b, i), nz))
            if op == "add" and out.lanes > 1:
                if a.id in self.unit and b.lanes == 1:
                    self.unit[out.id] = f"({self.unit[a.id]} + {self.name(b)})"
                elif b.id in self.unit and a.lanes == 1:
                    self.unit[out.id] = f"({self.name(a)} + {self.unit[b.id]})"
            return
        if op == "not":
            (x,) = args
            self._spmd_elementwise(out, lambda i: f"(!{self.lane(x, i)})")
            return
        if op == "where":
            c, a, b = args
            self._spmd_elementwise(out, lambda i: f"({self.lane(c, i)} ? {self.lane(a, i)} : {self.lane(b, i)})")
            return
        if op == "cast":
            x, dst = args
            self._spmd_elementwise(out, lambda i: _cast_expr(self.lane(x, i), x.dtype, dst))
            return
        if op == "fma":
            x, y, z = args
            self._spmd_elementwise(out, lambda i: _fma_expr(out.dtype, self.lane(x, i), self.lane(y, i),
                                                            self.lane(z, i)))
            return
        if op == "load":
            self._spmd_load(inst)
            return
        if op == "store":
            self._spmd_store(inst)
            return
        if op == "barrier":
            self.emit("__syncthreads();")
            return
        raise ValueError(f"unsupported op in spmd codegen: {op!r}")

    def _lane_mask(self, mask: ValueRef, i: int | str) -> str:
        m = "true" if self.is_const_true(mask) else self.lane(mask, str(i))
        if self.lane_guard:
            m = f"(eas_lv[{i}] && {m})" if m != "true" else f"eas_lv[{i}]"
        return m

    def _vector_ok(self, buf: ValueRef, off: ValueRef) -> bool:
        return (self.V == 4 and off.lanes > 1 and off.id in self.unit and buf.id in self.arg_c
                and not self.checked)

    def _spmd_load(self, inst: Inst) -> None:
        buf, off, mask = inst.args
        out = inst.out
        bn = self.name(buf)
        z = _zero(out.dtype)
        if out.lanes == 1:
            m = "true" if self.is_const_true(mask) else self.name(mask)
            m = self.both(m, self.inb(buf, self.name(off)))
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {m} ? {bn}[{self.name(off)}] : {z};")
            return
        self.emit(self._vec_decl(out))
        if self._vector_ok(buf, off):
            base = self.unit[off.id]
            vt, bytes_ = ("float4", 16) if out.dtype == DType.F32 else ("eas_h4", 8)
            self.emit("{")
            self.emit(f"const uint32_t eas_b = {base};", 2)
            self.emit(f"const bool eas_al = ((eas_b & 3u) == 0u) && ((((uint64_t){bn}) & {bytes_ - 1}ull) == 0ull);", 2)
            for j in range(self.J):
                ms = [self._lane_mask(mask, j * 4 + e) for e in range(4)]
                allm = " && ".join(ms)
                i0 = j * 4
                self.emit(f"if (eas_al && {allm}) {{", 2)
                self.emit(f"const {vt} eas_v = *reinterpret_cast<const {vt}*>({bn} + {self.lane(off, str(i0))});", 3)
                for e, comp in enumerate("xyzw"):
                    self.emit(f"v{out.id}[{i0 + e}] = eas_v.{comp};", 3)
                self.emit("} else {", 2)
                for e in range(4):
                    i = i0 + e
                    self.emit(f"v{out.id}[{i}] = {ms[e]} ? {bn}[{self.lane(off, str(i))}] : {z};", 3)
                self.emit("}", 2)
            self.emit("}")
            return
        for i in range(self.L):
            o = self.lane(off, str(i))
            m = self.both(self._lane_mask(mask, i), self.inb(buf, o))
            self.emit(f"v{out.id}[{i}] = {m} ? {bn}[{o}] : {z};")

    def _spmd_store(self, inst: Inst) -> None:
        buf, off, val, mask = inst.args
        bn = self.name(buf)
        if off.lanes == 1:
            m = "true" if self.is_const_true(mask) else self.name(mask)
            m = self.both(m, self.inb(buf, self.name(off), store=True))
            self.emit(f"if (threadIdx.x == 0 && {m}) {bn}[{self.name(off)}] = {self.name(val)};")
            return
        if self._vector_ok(buf, off):
            base = self.unit[off.id]
            vt, bytes_ = ("float4", 16) if buf.dtype == DType.F32 else ("eas_h4", 8)
            self.emit("{")
            self.emit(f"const uint32_t eas_b = {base};", 2)
            self.emit(f"const bool eas_al = ((eas_b & 3u) == 0u) && ((((uint64_t){bn}) & {bytes_ - 1}ull) == 0ull);", 2)
            for j in range(self.J):
                i0 = j * 4
                ms = [self._lane_mask(mask, i0 + e) for e in range(4)]
                self.emit(f"if (eas_al && {' && '.join(ms)}) {{", 2)
                vals = ", ".join(self.lane(val, str(i0 + e)) for e in range(4))
                self.emit(f"*reinterpret_cast<{vt}*>({bn} + {self.lane(off, str(i0))}) = {vt}{{{vals}}};", 3)
                self.emit("} else {", 2)
                for e in range(4):
                    i = i0 + e
                    self.emit(f"if ({ms[e]}) {bn}[{self.lane(off, str(i))}] = {self.lane(val, str(i))};", 3)
                self.emit("}", 2)
            self.emit("}")
            return
        for i in range(self.L):
            o = self.lane(off, str(i))
            m = self.both(self._lane_mask(mask, i), self.inb(buf, o, store=True))
            self.emit(f"if ({m}) {bn}[{o}] = {self.lane(val, str(i))};")

    @staticmethod
    def _const(dt: DType, v: Any) -> str:
        if dt == DType.BOOL:
            return "true" if v else "false"
        if dt == DType.U32:
            return f"{int(v) % (1 << 32)}u"
        if dt == DType.F32:
            return f32_literal(float(v))
        raise ValueError(f"unsupported const dtype {dt}")

    # ======================================================================
    # thread mode
    # ======================================================================
    def _thread(self) -> list[str]:
        self._smem_decls()
        self.emit("const uint32_t eas_gx = (blockIdx.x + eas_pid_x) * blockDim.x + threadIdx.x;")
        if self.cooperative:
            self.emit("const bool eas_on = eas_gx < eas_ntx;")
            self.ghost = "eas_on"
        else:
            self.emit("if (eas_gx >= eas_ntx) return;")
            self.ghost = None
        needs_lane = any(i.op in ("mma", "mma_store", "lane_id") for i in self.ir.insts)
        if needs_lane:
            self.emit("const uint32_t eas_lane = threadIdx.x & 31u;")
        groups = self._dot_groups()
        insts = self.ir.insts
        runs = []
        if os.environ.get("EAS_REROLL", "1") != "0":
            runs = find_runs(insts, keep_together=tuple(frozenset(m) for m in groups.values() if m))
        run_at = {r.first[0]: r for r in runs}
        in_run: set[int] = set()
        for r in runs:
            in_run |= r.ir_span
        for inst in insts:  # constants first: re-rolled blocks read them from any position
            if inst.op == "const":
                self._thread_inst(inst)
        for k, inst in enumerate(insts):
            if inst.op == "const":
                continue
            if k in run_at:
                self._emit_run(run_at[k], lambda body, r=run_at[k]: self._thread_block(r, body, groups))
            if k in in_run:
                continue
            if k in groups:
                if groups[k]:
                    self._dot_group([insts[j] for j in groups[k]])
                continue
            self._thread_inst(inst)
        return self.lines

    def _thread_block(self, run: Run, body: dict[int, Inst], groups: dict[int, list[int]]) -> None:
        for k in run.first:
            if k in groups:
                if groups[k]:
                    self._dot_group([body[j] for j in groups[k]])
                continue
            self._thread_inst(body[k])

    def _emit_run(self, run: Run, emit_body: Any) -> None:
        """Print a run of identical unrolled blocks as one loop over block 0 (bit-identical: the same
        operations in the same order).  Loop-carried operands live in mutable variables (lane arrays
        in SPMD mode) updated at the end of each iteration; the last iteration's values read after
        the loop are copied out.  ``emit_body(body)`` prints block 0 with ``body`` = {IR index:
        instruction with the carried and affine operands substituted}."""
        insts = self.ir.insts
        n = len(self.lines)
        rv = f"eas_r{n}"
        fresh = 1 << 40

        def declare(var: str, out: ValueRef, init: str | None) -> None:
            t = ctype(out.dtype)
            if out.lanes > 1:
                self.emit(f"{t} {var}[{self.L}];")
                if init is not None:
                    for i in range(self.L):
                        self.emit(f"{var}[{i}] = {init}[{i}];")
            else:
                self.emit(f"{t} {var}" + (f" = {init};" if init is not None else ";"))

        def copy(dst: str, src: str, lanes: int) -> None:
            if lanes > 1:
                for i in range(self.L):
                    self.emit(f"{dst}[{i}] = {src}[{i}];")
            else:
                self.emit(f"{dst} = {src};")

        body: dict[int, Inst] = {}
        carries: dict[str, int] = {}  # variable -> q
        for j, k in enumerate(run.first):
            inst = insts[k]
            args = list(inst.args)
            for a_i, f in enumerate(run.forms[j]):
                a = args[a_i]
                if f[0] == "carry":
                    _, q, init = f
                    var = f"eas_c{n}_{q}_{init}"
                    if var not in carries:
                        carries[var] = q
                        declare(var, insts[run.first[q]].out, self.name(a))
                    fresh += 1
                    self.alias[fresh] = var
                    args[a_i] = ValueRef(fresh, a.dtype, a.lanes)
                elif f[0] == "affine":
                    _, c0, d = f
                    fresh += 1
                    self.alias[fresh] = f"({c0 % (1 << 32)}u + {rv} * {d}u)"
                    args[a_i] = ValueRef(fresh, a.dtype, a.lanes)
            body[k] = Inst(inst.op, inst.out, tuple(args))
        escapes = {}
        for q in run.escapes:
            o = insts[run.first[q]].out
            self.uses[o.id] = max(1, self.uses.get(o.id, 0))
            escapes[q] = f"eas_e{n}_{q}"
            declare(escapes[q], o, None)
        self.emit(f"for (uint32_t {rv} = 0u; {rv} < {run.count}u; ++{rv}) {{")
        self.depth += 1
        emit_body(body)
        for var, q in carries.items():
            o = insts[run.first[q]].out
            copy(var, f"v{o.id}", o.lanes)
        for q, var in escapes.items():
            o = insts[run.first[q]].out
            copy(var, f"v{o.id}", o.lanes)
        self.depth -= 1
        self.emit("}")
        for q, var in escapes.items():
            o = insts[run.first[q]].out
            if o.lanes > 1:
                self.emit(f"{ctype(o.dtype)} v{run.last_out[q]}[{self.L}];")
                copy(f"v{run.last_out[q]}", var, o.lanes)
            else:
                self.emit(f"const {ctype(o.dtype)} v{run.last_out[q]} = {var};")

    _PURE = frozenset({"const", "add", "mul", "floordiv", "mod", "lt", "and", "or", "not", "where", "cast", "fma",
                       "program_id", "thread_id", "local_id", "lane_id", "sg_id", "tid"})

    def _dot_groups(self) -> dict[int, list[int]]:
        """Dots sharing (A buffer, A base, A stride, B buffer, B stride, K), up to 8, separated only by
        pure instructions that do not read them; {index of last member: members, other members: []}."""
        insts = self.ir.insts
        out: dict[int, list[int]] = {}
        taken: set[int] = set()
        if self.checked:
            return out

        def sig(i: Inst) -> tuple[int, ...]:
            a_buf, a_base, a_stride, b_buf, _b_base, b_stride, k = i.args
            return (a_buf.id, a_base.id, a_stride.id, b_buf.id, b_stride.id, k.id)

        for i, inst in enumerate(insts):
            if inst.op != "dot" or i in taken:
                continue
            members = [i]
            outs = {inst.out.id}
            s0 = sig(inst)
            for j in range(i + 1, min(len(insts), i + 64)):
                nxt = insts[j]
                if nxt.op == "dot" and sig(nxt) == s0 and len(members) < 8:
                    members.append(j)
                    outs.add(nxt.out.id)
                    continue
                if nxt.op in self._PURE and not any(isinstance(a, ValueRef) and a.id in outs for a in nxt.args):
                    continue
                break
            if len(members) > 1:
                for m in members:
                    taken.add(m)
                    out[m] = []
                out[members[-1]] = members
        return out

    def _dot_group(self, dots: list[Inst]) -> None:
        """One k loop for several dots: A is loaded once per k; when four B bases are X+0..3 the
        four B values come from one vector load whenever that address is aligned.  Each dot keeps
        its own strict k-order fma chain, so results equal the separate loops bit for bit."""
        a_buf, a_base, a_stride, b_buf, _bb, b_stride, k_ref = dots[0].args
        outs = [d.out.id for d in dots]
        for o in outs:
            self.emit(f"float v{o} = 0.0f;")
        # vector candidate: first four members with B base = X + 0, 1, 2, 3
        vec = None
        if len(dots) >= 4:
            bases = []
            for d in dots[:4]:
                bref = d.args[4]
                bd = self.defs.get(bref.id)
                if bd is not None and bd.op == "add":
                    x, y = bd.args
                    cy, cx = self.defs.get(y.id), self.defs.get(x.id)
                    if cy is not None and cy.op == "const" and cy.out.dtype == DType.U32:
                        bases.append((x.id, int(cy.args[0]), bref))
                        continue
                    if cx is not None and cx.op == "const" and cx.out.dtype == DType.U32:
                        bases.append((y.id, int(cx.args[0]), bref))
                        continue
                bases.append((bref.id, 0, bref))
            if len({b[0] for b in bases}) == 1 and [b[1] for b in bases] == [0, 1, 2, 3]:
                vec = bases[0][2]
        guard = self._guard("true")
        self.emit("{" if guard == "true" else f"if ({guard}) {{")
        self.emit(f"uint32_t eas_ai = {self.name(a_base)};", 2)
        for n, d in enumerate(dots):
            self.emit(f"uint32_t eas_bi{n} = {self.name(d.args[4])};", 2)
        kd = self.defs.get(k_ref.id)
        if kd is not None and kd.op == "const" and 1 <= int(kd.args[0]) <= 32:
            self.emit("#pragma unroll 4", 2)
        self.emit(f"for (uint32_t eas_k = 0; eas_k < {self.name(k_ref)}; ++eas_k) {{", 2)
        A, B = self.name(a_buf), self.name(b_buf)
        self.emit(f"const float eas_av = {_as_float(a_buf.dtype, f'{A}[eas_ai]')};", 3)

        def scalar(n: int, o: int) -> str:
            return f"v{o} = fmaf(eas_av, {_as_float(b_buf.dtype, f'{B}[eas_bi{n}]')}, v{o});"

        if vec is not None:
            vt, comps = ("float4", "xyzw") if b_buf.dtype == DType.F32 else ("eas_h4", "xyzw")
            self.emit("if ((eas_bi0 & 3u) == 0u) {", 3)
            self.emit(f"const {vt} eas_bv = *reinterpret_cast<const {vt}*>({B} + eas_bi0);", 4)
            for n in range(4):
                self.emit(f"v{outs[n]} = fmaf(eas_av, {_as_float(b_buf.dtype, f'eas_bv.{comps[n]}')}, v{outs[n]});", 4)
            self.emit("} else {", 3)
            for n in range(4):
                self.emit(scalar(n, outs[n]), 4)
            self.emit("}", 3)
            for n in range(4, len(dots)):
                self.emit(scalar(n, outs[n]), 3)
        else:
            for n, o in enumerate(outs):
                self.emit(scalar(n, o), 3)
        self.emit(f"eas_ai += {self.name(a_stride)};" + "".join(f" eas_bi{n} += {self.name(b_stride)};"
                                                             for n in range(len(dots))), 3)
        self.emit("}", 2)
        self.emit("}")

    def _guard(self, cond: str) -> str:
        if self.ghost is None:
            return cond
        return self.ghost if cond == "true" else f"({self.ghost} && {cond})"

    def _thread_inst(self, inst: Inst) -> None:
        op, out, args = inst.op, inst.out, inst.args
        if op in ("arg", "alloc_tg"):
            return
        if out is not None and self.uses.get(out.id, 0) == 0 and op not in ("store", "mma_store"):
            return  # e.g. the tid that only defines BLOCK
        if op == "const":
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {self._const(out.dtype, args[0])};")
        elif op == "program_id":
            ax = "xyz"[int(args[0])]
            self.emit(f"const uint32_t v{out.id} = blockIdx.{ax} + eas_pid_{ax};")
        elif op == "thread_id":
            ax = int(args[0])
            if ax == 0:
                self.emit(f"const uint32_t v{out.id} = eas_gx;")
            else:
                a = "xyz"[ax]
                self.emit(f"const uint32_t v{out.id} = blockIdx.{a} + eas_pid_{a};")
        elif op == "local_id":
            self.emit(f"const uint32_t v{out.id} = {'threadIdx.x' if int(args[0]) == 0 else '0u'};")
        elif op == "lane_id":
            self.emit(f"const uint32_t v{out.id} = eas_lane;")
        elif op == "sg_id":
            self.emit(f"const uint32_t v{out.id} = threadIdx.x >> 5;")
        elif op == "tid":
            self.emit(f"const uint32_t v{out.id} = {int(args[0])}u + threadIdx.x;")
        elif op == "arange":
            raise ValueError("arange is not supported in thread mode codegen; use mk.tid(...) for thread-level kernels")
        elif op in ("add", "mul", "floordiv", "mod", "lt", "and", "or"):
            a, b = args
            expr = _binop_expr(op, a.dtype, self.name(a), self.name(b), self._nonzero_const(b))
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {expr};")
        elif op == "not":
            self.emit(f"const bool v{out.id} = !{self.name(args[0])};")
        elif op == "where":
            c, a, b = args
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {self.name(c)} ? {self.name(a)} : {self.name(b)};")
        elif op == "cast":
            x, dst = args
            self.emit(f"const {ctype(out.dtype)} v{out.id} = {_cast_expr(self.name(x), x.dtype, dst)};")
        elif op == "fma":
            x, y, z = args
            self.emit(f"const {ctype(out.dtype)} v{out.id} = "
                      f"{_fma_expr(out.dtype, self.name(x), self.name(y), self.name(z))};")
        elif op == "load":
            buf, off, mask = args
            m = self._guard("true" if self.is_const_true(mask) else self.name(mask))
            m = self.both(m, self.inb(buf, self.name(off)))
            rhs = f"{self.name(buf)}[{self.name(off)}]"
            if m == "true":
                self.emit(f"const {ctype(out.dtype)} v{out.id} = {rhs};")
            else:
                self.emit(f"const {ctype(out.dtype)} v{out.id} = {m} ? {rhs} : {_zero(out.dtype)};")
        elif op == "store":
            buf, off, val, mask = args
            m = self._guard("true" if self.is_const_true(mask) else self.name(mask))
            m = self.both(m, self.inb(buf, self.name(off), store=True))
            st = f"{self.name(buf)}[{self.name(off)}] = {self.name(val)};"
            self.emit(st if m == "true" else f"if ({m}) {st}")
        elif op == "barrier":
            self.emit("__syncthreads();")
        elif op == "dot":
            self._dot(inst)
        elif op == "mma_zero":
            self.emit(f"float2 v{out.id} = make_float2(0.0f, 0.0f);")
        elif op == "mma":
            self._mma(inst)
        elif op == "mma_store":
            buf, base, stride, frag = args
            g = self._guard("true")
            b, s, f = self.name(base), self.name(stride), self.name(frag)
            self.emit("{")
            self.emit(f"const uint32_t eas_o = {b} + (eas_lane >> 2) * {s} + (eas_lane & 3u) * 2u;", 2)
            if self.checked:
                for e, comp in ((("eas_o"), "x"), (("eas_o + 1u"), "y")):
                    self.emit(f"if ({self.both(g, self.inb(buf, e, store=True))}) {self.name(buf)}[{e}] = {f}.{comp};", 2)
            else:
                pre = "" if g == "true" else f"if ({g}) "
                self.emit(f"{pre}{{ {self.name(buf)}[eas_o] = {f}.x; {self.name(buf)}[eas_o + 1u] = {f}.y; }}", 2)
            self.emit("}")
        else:
            raise ValueError(f"unsupported op: {op}")

    def _dot(self, inst: Inst) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, k_ref = inst.args
        o = inst.out.id
        kd = self.defs.get(k_ref.id)
        unroll = "#pragma unroll" if kd is not None and kd.op == "const" and 1 <= int(kd.args[0]) <= 32 else ""
        self.emit(f"float v{o} = 0.0f;")
        body_guard = self._guard("true")
        self.emit("{" if body_guard == "true" else f"if ({body_guard}) {{")
        self.emit(f"uint32_t eas_ai = {self.name(a_base)}, eas_bi = {self.name(b_base)};", 2)
        if unroll:
            self.emit(unroll, 2)
        self.emit(f"for (uint32_t eas_k = 0; eas_k < {self.name(k_ref)}; ++eas_k) {{", 2)
        av = _as_float(a_buf.dtype, self.ld(a_buf, "eas_ai"))
        bv = _as_float(b_buf.dtype, self.ld(b_buf, "eas_bi"))
        self.emit(f"v{o} = fmaf({av}, {bv}, v{o});", 3)
        self.emit(f"eas_ai += {self.name(a_stride)}; eas_bi += {self.name(b_stride)};", 3)
        self.emit("}", 2)
        self.emit("}")

    def _mma(self, inst: Inst) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, acc = inst.args
        o = inst.out.id
        A, B = self.name(a_buf), self.name(b_buf)
        ab, as_, bb, bs = self.name(a_base), self.name(a_stride), self.name(b_base), self.name(b_stride)
        on = self._guard("true")
        self.emit(f"float2 v{o};")
        self.emit("{")
        self.emit("const uint32_t eas_g = eas_lane >> 2, eas_t = eas_lane & 3u;", 2)
        if a_buf.dtype == DType.F16 and b_buf.dtype == DType.F16:
            ai = f"{ab} + eas_g * {as_} + eas_t * 2u"
            bi0 = f"{bb} + (eas_t * 2u) * {bs} + eas_g"
            a0, a1 = self.ld(a_buf, f"({ai})"), self.ld(a_buf, f"({ai} + 1u)")
            b0, b1 = self.ld(b_buf, f"({bi0})"), self.ld(b_buf, f"({bi0} + {bs})")
            if on == "true":
                self.emit(f"const uint32_t eas_a = eas_pack2({a0}, {a1});", 2)
                self.emit(f"const uint32_t eas_b = eas_pack2({b0}, {b1});", 2)
            else:
                self.emit(f"const uint32_t eas_a = {on} ? eas_pack2({a0}, {a1}) : 0u;", 2)
                self.emit(f"const uint32_t eas_b = {on} ? eas_pack2({b0}, {b1}) : 0u;", 2)
            self.emit(f"v{o} = eas_mma_f16(eas_a, eas_b, {self.name(acc)});", 2)
        else:
            self.emit(f"float eas_d0 = {self.name(acc)}.x, eas_d1 = {self.name(acc)}.y;", 2)
            pre = "" if on == "true" else f"if ({on}) "
            self.emit(f"{pre}{{", 2)
            self.emit("#pragma unroll", 3)
            self.emit("for (uint32_t eas_k = 0; eas_k < 8u; ++eas_k) {", 3)
            av = _as_float(a_buf.dtype, self.ld(a_buf, f"({ab} + eas_g * {as_} + eas_k)"))
            b0 = _as_float(b_buf.dtype, self.ld(b_buf, f"({bb} + eas_k * {bs} + eas_t * 2u)"))
            b1 = _as_float(b_buf.dtype, self.ld(b_buf, f"({bb} + eas_k * {bs} + eas_t * 2u + 1u)"))
            self.emit(f"const float eas_av = {av};", 4)
            self.emit(f"eas_d0 = fmaf(eas_av, {b0}, eas_d0); eas_d1 = fmaf(eas_av, {b1}, eas_d1);", 4)
            self.emit("}", 3)
            self.emit("}", 2)
            self.emit(f"v{o} = make_float2(eas_d0, eas_d1);", 2)
        self.emit("}")


@dataclass(frozen=True, slots=True)
class ElementwiseInfo:
    """Every memory access of the kernel is at the global element index X (= program_id(0)*BLOCK +
    lane/thread), masked by ``X < bound`` or not at all.  Program p then touches only elements
    [p*BLOCK, p*BLOCK + BLOCK), so any split of the programs splits the buffers the same way."""

    block: int
    reads: frozenset[str]                 # buffer args that are loaded
    writes: frozenset[str]                # buffer args that are stored
    store_bounds: tuple[tuple[str, Any], ...]  # (buffer, bound): ("arg", name), ("const", v) or None (unmasked)


def elementwise_info(ir: IRModule, block: int, mode: str) -> ElementwiseInfo | None:
    defs = {i.out.id: i for i in ir.insts if i.out is not None}
    if any(i.op in ("program_id", "thread_id") and int(i.args[0]) != 0 for i in ir.insts):
        return None
    if any(i.op in ("dot", "mma", "mma_store", "alloc_tg", "barrier", "local_id", "lane_id", "sg_id") for i in ir.insts):
        return None

    def op(ref: ValueRef) -> Inst | None:
        return defs.get(ref.id)

    def is_const(ref: ValueRef, v: int) -> bool:
        d = op(ref)
        return d is not None and d.op == "const" and not isinstance(d.args[0], bool) and int(d.args[0]) == v

    def is_index(ref: ValueRef) -> bool:
        d = op(ref)
        if d is None:
            return False
        if mode == "thread" and d.op == "thread_id":
            return True
        if d.op != "add":
            return False
        for x, y in (d.args, d.args[::-1]):
            dx, dy = op(x), op(y)
            if dx is None or dy is None or dx.op != "mul":
                continue
            local_ok = (dy.op == "arange" if mode == "spmd" else dy.op == "tid") and tuple(
                int(v) for v in dy.args) == (0, block)
            p, q = dx.args
            pid_ok = any((op(u) is not None and op(u).op == "program_id" and is_const(w, block))
                         for u, w in ((p, q), (q, p)))
            if local_ok and pid_ok:
                return True
        return False

    def bound(mask: ValueRef, idx: ValueRef) -> Any:
        d = op(mask)
        if d is not None and d.op == "const" and d.args[0] is True:
            return None
        if d is not None and d.op == "lt" and d.args[0].id == idx.id:
            b = op(d.args[1])
            if b is not None and b.op == "arg":
                return ("arg", str(b.args[0]))
            if b is not None and b.op == "const" and not isinstance(b.args[0], bool):
                return ("const", int(b.args[0]))
        return "bad"

    arg_names = {i.out.id: str(i.args[0]) for i in ir.insts if i.op == "arg"}
    reads, writes, bounds = set(), set(), []
    for inst in ir.insts:
        if inst.op not in ("load", "store"):
            continue
        buf, off = inst.args[0], inst.args[1]
        mask = inst.args[2] if inst.op == "load" else inst.args[3]
        if buf.id not in arg_names or not is_index(off):
            return None
        b = bound(mask, off)
        if b == "bad":
            return None
        name = arg_names[buf.id]
        if inst.op == "load":
            reads.add(name)
        else:
            if inst.args[2].lanes not in (1, off.lanes):
                return None
            writes.add(name)
            bounds.append((name, b))
    if not writes:
        return None
    return ElementwiseInfo(block, frozenset(reads), frozenset(writes), tuple(bounds))


def ir_to_cuda(ir: IRModule, checked: bool | None = None) -> Lowered:
    """Lower validated, optimised IR to one CUDA kernel (plus an optional native plan).

    ``checked`` (default: ``EAS_BOUNDS_CHECK``) lowers with per-access bounds checks; such a kernel
    always runs as generated (no native plan) and is not split by the host pipelines."""
    if checked is None:
        checked = bounds_check_enabled()
    lowered = _Emitter(ir, checked).run()
    if checked:
        from ..analysis import infer_reads

        lowered.reads = infer_reads(ir)
        return lowered
    from .patterns import match_native

    lowered.native = match_native(ir, lowered)
    lowered.elementwise = elementwise_info(ir, lowered.block_size, lowered.mode)
    from ..analysis import infer_reads

    lowered.reads = infer_reads(ir)
    return lowered
