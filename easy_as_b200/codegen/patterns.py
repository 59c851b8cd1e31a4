"""Recognise IR shapes that map onto hand-written native kernels.

``match_native(ir, lowered)`` returns a plan with
``try_launch(runtime, ck, runtime_args, args, device, stream, programs, ntx)``,
or None.  A plan launches its native kernel only when the launch-time values
fit it and returns False otherwise; the generic NVRTC kernel then runs.  Both
compute the same IR.

Dot-GEMM pattern (the fp16 ``mk.dot`` GEMM of configs C4/C5)
-------------------------------------------------------------
A thread-mode kernel whose only memory operations are one ``dot`` over two f16
*global* buffers and one store of that dot's f32 result into a global f32
buffer, with every index an affine function of the launch coordinates

    X = program_id(0) * BLOCK + tid,  Y = program_id(1),  Z = program_id(2)

(coefficients may be products of scalar arguments and constants), and a store
mask that is a conjunction of ``coordinate < bound`` tests.  Per launch, the
scalar values are substituted, each coordinate is classified by where it
appears (A only -> M, B only -> N, both -> batch), and the strides of
``A[b][m][k]``, ``B[b][k][n]`` and ``C[b][m][n]`` are read off the
coefficients.  The plan applies when A is K-major (``a_stride == 1``), B is
N-major or K-major, C is row-major, no u32 index computation of the IR can wrap
(interval check with the real scalar values), all reads stay inside the
buffers, and the TMA alignment rules hold.

The reference semantics of ``dot`` is a strictly ordered f32 ``fma`` chain
(easy_as ``eas/codegen/msl.py:920-952``); the tensor-core kernel sums the same
exact f16 products in f32 in a different order, so results agree within
f32 rounding (the parity tests use the fp16-GEMM tolerance).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Mapping

import numpy as np

from ..ir import DType, IRModule

Mono = tuple[str, ...]          # sorted symbol names; () is the constant term
Poly = dict[Mono, int]          # monomial -> integer coefficient

COORDS = ("P0", "P1", "P2", "T")
U32_LIMIT = 1 << 32


def _padd(a: Poly, b: Poly) -> Poly:
    out = dict(a)
    for m, c in b.items():
        out[m] = out.get(m, 0) + c
    return {m: c for m, c in out.items() if c}


def _pmul(a: Poly, b: Poly) -> Poly:
    out: Poly = {}
    for ma, ca in a.items():
        for mb, cb in b.items():
            m = tuple(sorted(ma + mb))
            out[m] = out.get(m, 0) + ca * cb
    return {m: c for m, c in out.items() if c}


def _peval(p: Poly, scalars: dict[str, int]) -> dict[str, int] | None:
    """Substitute scalar values; result is linear {coord or '': coeff}, or None if nonlinear."""
    out: dict[str, int] = {}
    for mono, c in p.items():
        coord = None
        v = c
        for s in mono:
            if s in COORDS:
                if coord is not None:
                    return None
                coord = s
            else:
                v *= scalars[s]
        key = coord or ""
        out[key] = out.get(key, 0) + v
    return out


@dataclass
class DotGemmPlan:
    """Native tcgen05 GEMM for the dot pattern (see module docstring)."""

    ir: IRModule
    block: int
    a_arg: str
    b_arg: str
    c_arg: str
    a_base: Poly
    b_base: Poly
    a_stride: Poly
    b_stride: Poly
    k: Poly
    c_off: Poly
    atoms: list[tuple[Poly, Poly]]   # mask: conjunction of lhs < rhs
    block_n: int
    kind: str = "dot_gemm_f16_tcgen05"
    last_reason: str = ""
    tile_m: int = 0      # 0: the library picks the M tile; 128: 1-SM kernel; 256: CTA pair
    block_k: int = 0     # 0 / 64: one 64-deep k-block per pipeline stage; 128: two
    _memo: dict = field(default_factory=dict, repr=False, compare=False)

    def apply_tile_hints(self, meta: Mapping[str, Any]) -> None:
        """Take the kernel's ``BLOCK_M`` / ``BLOCK_K`` constexprs, when it has them, as the native
        tile request (``eas_gemm_f16_tile``): the autotune space of a dot GEMM, in which the
        reference's Metal kernel uses the same names as threadgroup tile sizes.  Values other than
        128/256 (``BLOCK_M``) and 64/128 (``BLOCK_K``), 0 included, leave the choice to the library."""
        bm, bk = meta.get("BLOCK_M"), meta.get("BLOCK_K")
        self.tile_m = int(bm) if isinstance(bm, int) and bm in (128, 256) else 0
        self.block_k = int(bk) if isinstance(bk, int) and bk in (64, 128) else 0

    # -- launch-time mapping -------------------------------------------------
    def _coord_forms(self, forms: dict[str, dict[str, int]]) -> dict[str, dict[str, int]] | None:
        """Fold (P0, T) into X = P0*BLOCK + T; None if a form uses them otherwise."""
        out = {}
        for name, f in forms.items():
            t = f.get("T", 0)
            p0 = f.get("P0", 0)
            if p0 != t * self.block:
                return None
            out[name] = {"": f.get("", 0), "X": t, "Y": f.get("P1", 0), "Z": f.get("P2", 0)}
        return out

    def map_launch(self, scalars: dict[str, int], programs: tuple[int, int, int], ntx: int,
                   pid_base: tuple[int, int, int] = (0, 0, 0)) -> dict[str, Any] | None:
        """GEMM of the programs ``pid_base + [0, programs)`` (program ids offset per axis); memoised
        per launch values (the mapping is a pure function of them)."""
        key = (tuple(sorted(scalars.items())), tuple(programs), ntx, tuple(pid_base))
        hit = self._memo.get(key)
        if hit is None:
            m = self._map_launch(scalars, programs, ntx, pid_base)
            hit = (m, self.last_reason)
            if len(self._memo) >= 64:
                self._memo.clear()
            self._memo[key] = hit
        self.last_reason = hit[1]
        return hit[0]

    def _map_launch(self, scalars: dict[str, int], programs: tuple[int, int, int], ntx: int,
                    pid_base: tuple[int, int, int] = (0, 0, 0)) -> dict[str, Any] | None:
        polys = {"a": self.a_base, "b": self.b_base, "sa": self.a_stride, "sb": self.b_stride, "k": self.k,
                 "c": self.c_off}
        for i, (lhs, rhs) in enumerate(self.atoms):
            polys[f"l{i}"] = lhs
            polys[f"r{i}"] = rhs
        lin = {}
        for n, p in polys.items():
            e = _peval(p, scalars)
            if e is None:
                self.last_reason = "nonlinear index"
                return None
            lin[n] = e
        f = self._coord_forms(lin)
        if f is None:
            self.last_reason = "program_id(0) and tid not combined as program_id(0)*BLOCK + tid"
            return None
        for n in ("sa", "sb", "k"):
            if f[n]["X"] or f[n]["Y"] or f[n]["Z"]:
                self.last_reason = f"{n} depends on the thread coordinates"
                return None
        # program-id offsets: X = X' + base_x, Y = Y' + base_y, Z = Z' + base_z with X', Y', Z' from 0
        shift = {"X": pid_base[0] * self.block, "Y": pid_base[1], "Z": pid_base[2]}
        for form in f.values():
            form[""] += sum(form[c] * shift[c] for c in "XYZ")
        gx, gy, gz = programs
        ext = {"X": min(gx * self.block, ntx - shift["X"]), "Y": gy, "Z": gz}
        for i in range(len(self.atoms)):
            lhs, rhs = f[f"l{i}"], f[f"r{i}"]
            if rhs["X"] or rhs["Y"] or rhs["Z"]:
                self.last_reason = "mask bound depends on the thread coordinates"
                return None
            coords = [c for c in "XYZ" if lhs[c]]
            if len(coords) != 1 or lhs[coords[0]] != 1 or lhs[""] != shift[coords[0]]:
                self.last_reason = "mask is not coordinate < bound"
                return None
            ext[coords[0]] = min(ext[coords[0]], max(rhs[""] - lhs[""], 0))
        if min(ext.values()) <= 0:
            return {"empty": True}
        roles: dict[str, str] = {}
        for cc in "XYZ":
            if ext[cc] == 1:
                continue
            in_a, in_b = f["a"][cc] != 0, f["b"][cc] != 0
            role = "m" if in_a and not in_b else "n" if in_b and not in_a else "batch" if in_a and in_b else None
            if role is None or role in roles.values():
                self.last_reason = f"coordinate {cc} has no GEMM role"
                return None
            roles[cc] = role
        by_role = {r: c for c, r in roles.items()}

        def coef(form: str, role: str) -> int:
            c = by_role.get(role)
            return f[form][c] if c else 0

        def extent(role: str) -> int:
            c = by_role.get(role)
            return ext[c] if c else 1

        M, N, B = extent("m"), extent("n"), extent("batch")
        K = f["k"][""]
        sa, sb = f["sa"][""], f["sb"][""]
        if K <= 0 or sa != 1:
            self.last_reason = "K == 0 or A is not K-major"
            return None
        b_n = coef("b", "n")
        if b_n == 1 and (sb != 1 or N == 1):
            b_kmajor, ldb = 0, sb
        elif sb == 1:
            b_kmajor, ldb = 1, b_n
        else:
            self.last_reason = "B is neither N-major nor K-major"
            return None
        if N > 1 and coef("c", "n") != 1:
            self.last_reason = "C is not row-major"
            return None
        # C writes must be distinct per output element and rows must not overlap
        ldc, cbs = coef("c", "m"), coef("c", "batch")
        if (M > 1 and ldc < N) or (B > 1 and cbs < (M - 1) * ldc + N):
            self.last_reason = "C rows or batches overlap"
            return None
        lda, abs_ = coef("a", "m"), coef("a", "batch")
        bbs = coef("b", "batch")
        # largest index each address expression reaches (no u32 wrap allowed)
        top_a = f["a"][""] + lda * (M - 1) + abs_ * (B - 1) + (K - 1)
        top_b = f["b"][""] + (b_n * (N - 1) + bbs * (B - 1) + sb * (K - 1))
        top_c = f["c"][""] + ldc * (M - 1) + cbs * (B - 1) + (N - 1)
        if max(top_a, top_b, top_c) >= U32_LIMIT or not self._no_wrap(scalars, programs, pid_base):
            self.last_reason = "u32 index arithmetic would wrap"
            return None
        return {"M": M, "N": N, "K": K, "batch": B, "a0": f["a"][""], "b0": f["b"][""], "c0": f["c"][""],
                "lda": lda, "a_bs": abs_ if B > 1 else 0, "ldb": ldb, "b_bs": bbs if B > 1 else 0,
                "b_kmajor": b_kmajor, "ldc": ldc if M > 1 else N, "c_bs": cbs if B > 1 else 0,
                "top_a": top_a, "top_b": top_b, "top_c": top_c}

    def _no_wrap(self, scalars: dict[str, int], programs: tuple[int, int, int],
                 pid_base: tuple[int, int, int] = (0, 0, 0)) -> bool:
        """Interval upper bounds of every u32 node stay below 2**32 for this launch."""
        hi: dict[int, int] = {}
        gx, gy, gz = (b + n for b, n in zip(pid_base, programs))
        for inst in self.ir.insts:
            o = inst.out
            if o is None or o.dtype != DType.U32:
                continue
            op, a = inst.op, inst.args
            if op == "arg":
                hi[o.id] = int(scalars[f"${a[0]}"])
            elif op == "const":
                hi[o.id] = int(a[0])
            elif op == "program_id":
                hi[o.id] = (gx, gy, gz)[int(a[0])] - 1
            elif op == "thread_id":
                hi[o.id] = gx * self.block - 1 if int(a[0]) == 0 else (gx, gy, gz)[int(a[0])] - 1
            elif op in ("tid",):
                hi[o.id] = int(a[0]) + self.block - 1
            elif op == "local_id":
                hi[o.id] = self.block - 1
            elif op == "add":
                hi[o.id] = hi[a[0].id] + hi[a[1].id]
            elif op == "mul":
                hi[o.id] = hi[a[0].id] * hi[a[1].id]
            elif op == "where":
                hi[o.id] = max(hi[a[1].id], hi[a[2].id])
            else:
                return False
            if hi[o.id] >= U32_LIMIT:
                return False
        return True

    def _restage(self, rt: Any, lib: Any, m: dict[str, Any], a: int, b: int, device: int,
                 stream: int) -> tuple[int, int, int, int, int, int, list] | None:
        """A and B as the tcgen05 kernel will read them: in place when TMA can (16-byte aligned base
        and pitches), else re-pitched into scratch rows padded to 8 elements (the GEMM still reads
        only K columns of A and K rows or columns of B, so the padding never enters a sum)."""
        M, N, K, B = m["M"], m["N"], m["K"], m["batch"]
        lda, a_bs, ldb, b_bs = m["lda"], m["a_bs"], m["ldb"], m["b_bs"]
        keep: list = []
        if not _tma_rows_ok(a, lda, a_bs, B):
            got = _restage_operand(rt, lib, a, M, K, lda, a_bs, B, device, stream, "dot_a16")
            if got is None:
                self.last_reason = "A re-pitch scratch unavailable (CUDA-graph capture)"
                return None
            a, lda, a_bs, owner = got
            keep.append(owner)
        if not _tma_rows_ok(b, ldb, b_bs, B):
            rows, cols = (N, K) if m["b_kmajor"] else (K, N)
            got = _restage_operand(rt, lib, b, rows, cols, ldb, b_bs, B, device, stream, "dot_b16")
            if got is None:
                self.last_reason = "B re-pitch scratch unavailable (CUDA-graph capture)"
                return None
            b, ldb, b_bs, owner = got
            keep.append(owner)
        return a, lda, a_bs if B > 1 else 0, b, ldb, b_bs if B > 1 else 0, keep

    def covers(self, runtime_args: dict[str, Any], programs: tuple[int, int, int], ntx: int, name: str,
               numel: int) -> bool:
        """True when this launch stores every element of buffer ``name`` (numel elements from index 0):
        the output rectangle M x N of every batch is one dense block starting at 0.  A property of
        the kernel's stores, so it holds whichever kernel runs the launch."""
        if name != self.c_arg:
            return False
        scalars = {f"${a.name}": int(runtime_args[a.name]) for a in self.ir.args if a.kind == "scalar"}
        m = self.map_launch(scalars, programs, ntx)
        if m is None or m.get("empty"):
            return False
        M, N, B = m["M"], m["N"], m["batch"]
        dense = (M == 1 or m["ldc"] == N) and (B == 1 or m["c_bs"] == M * N)
        return dense and m["c0"] == 0 and M * N * B == numel

    # -- launch ------------------------------------------------------------------
    def try_launch(self, rt: Any, ck: Any, runtime_args: dict[str, Any], args: dict[str, Any], device: int,
                   stream: int, programs: tuple[int, int, int], ntx: int, pid_base: tuple[int, int, int] = (0, 0, 0),
                   elem_base: dict[str, int] | None = None) -> bool:
        """Launch the native kernel for programs ``pid_base + [0, programs)``; buffers listed in
        ``elem_base`` hold only the elements from that global index on (their pointers are already
        moved back by it)."""
        import os

        if os.environ.get("EAS_DISABLE_NATIVE", "0") not in ("", "0"):
            self.last_reason = "disabled by EAS_DISABLE_NATIVE"
            return False
        scalars = {f"${a.name}": int(runtime_args[a.name]) for a in self.ir.args if a.kind == "scalar"}
        m = self.map_launch(scalars, programs, ntx, pid_base)
        if m is None:
            return False
        if m.get("empty"):
            return True
        eb = elem_base or {}
        for name, lo, top in ((self.a_arg, m["a0"], m["top_a"]), (self.b_arg, m["b0"], m["top_b"]),
                              (self.c_arg, m["c0"], m["top_c"])):
            e = int(eb.get(name, 0))
            if lo < e or top >= e + _numel(runtime_args[name]):
                self.last_reason = "operand extents exceed the buffers"
                return False
        a = args[self.a_arg].ptr + 2 * m["a0"]
        b = args[self.b_arg].ptr + 2 * m["b0"]
        c = args[self.c_arg].ptr + 4 * m["c0"]
        lib = rt.lib()
        staged = self._restage(rt, lib, m, a, b, device, stream)
        if staged is None:
            return False
        a, lda, a_bs, b, ldb, b_bs, _keep = staged
        rc = lib.eas_gemm_f16_tile(a, b, c, m["M"], m["N"], m["K"], m["batch"], lda, a_bs, ldb, b_bs,
                                   m["b_kmajor"], m["ldc"], m["c_bs"], self.tile_m, self.block_n, self.block_k, stream)
        if rc == 4:  # EAS_ERR_VALUE: layout the native kernel does not take (alignment, sizes)
            from ..runtime import cuda_ext

            self.last_reason = cuda_ext.last_error()
            return False
        from ..runtime import cuda_ext

        cuda_ext.check(rc, "gemm_f16 (tcgen05)")
        rt.launch_count += 1
        rt.native_launches += 1
        return True


def _tma_rows_ok(ptr: int, ld: int, bs: int, batch: int) -> bool:
    """f16 rows TMA reads in place: 16-byte aligned base, row and batch pitches multiples of 8 elements."""
    return ptr % 16 == 0 and ld % 8 == 0 and (batch == 1 or bs % 8 == 0)


def _restage_operand(rt: Any, lib: Any, ptr: int, rows: int, cols: int, ld: int, bs: int, batch: int, device: int,
                     stream: int, tag: str) -> tuple[int, int, int, Any] | None:
    """Copy f16 rows [batch][rows][cols] (pitch ld, batch pitch bs) to scratch rows padded to a
    multiple of 8 elements (``eas_pad_f16_2d``); (pointer, ld', bs', owner) or None when no scratch
    can be had (inside a CUDA-graph capture without torch)."""
    from ..runtime import cuda_ext

    cols_pad = -(-cols // 8) * 8
    got = rt.scratch(device, stream, tag, 2 * batch * rows * cols_pad)
    if got is None:
        return None
    dst, owner = got
    cuda_ext.check(lib.eas_pad_f16_2d(ptr, dst, rows, cols_pad, ld, cols_pad, rows, cols, batch, bs, rows * cols_pad,
                                      stream), f"re-pitch {tag}")
    rt.launch_count += 1
    return dst, cols_pad, rows * cols_pad, owner


def _numel(v: Any) -> int:
    if type(v) is np.ndarray:
        return int(v.size)
    if getattr(v, "__eas_tensor__", False):
        return int(v.nbytes) // v.dtype.itemsize
    if hasattr(v, "numel") and callable(v.numel):
        return int(v.numel())
    if hasattr(v, "size") and isinstance(v.size, int):
        return int(v.size)
    n = 1
    for d in getattr(v, "shape", (1,)):
        n *= int(d)
    return n


# ---------------------------------------------------------------------------
# static matching
# ---------------------------------------------------------------------------

_ALLOWED = {"arg", "const", "program_id", "thread_id", "tid", "local_id", "add", "mul", "lt", "and", "where", "dot",
            "store"}


def _match_dot_gemm(ir: IRModule, lowered: Any) -> DotGemmPlan | None:
    if lowered.mode != "thread":
        return None
    if any(i.op not in _ALLOWED for i in ir.insts):
        return None
    dots = [i for i in ir.insts if i.op == "dot"]
    stores = [i for i in ir.insts if i.op == "store"]
    if len(dots) != 1 or len(stores) != 1:
        return None
    dot, st = dots[0], stores[0]
    buf, off, val, mask = st.args
    if val.id != dot.out.id or val.lanes != 1:
        return None
    arg_names = {i.out.id: str(i.args[0]) for i in ir.insts if i.op == "arg"}
    a_buf, a_base, a_stride, b_buf, b_base, b_stride, k = dot.args
    if not all(x.id in arg_names for x in (a_buf, b_buf, buf)):
        return None
    defs = {i.out.id: i for i in ir.insts if i.out is not None}
    # `where(store_mask, K, 0)` as the dot length: threads outside C read nothing,
    # threads inside use K -- the same sums the native kernel computes
    kd = defs.get(k.id)
    if kd is not None and kd.op == "where":
        c_, k_in, zero = kd.args
        zd = defs.get(zero.id)
        if c_.id != mask.id or zd is None or zd.op != "const" or zd.args[0] != 0:
            return None
        k = k_in
    if any(i.op == "where" and i.out.dtype != DType.U32 for i in ir.insts):
        return None
    if a_buf.dtype != DType.F16 or b_buf.dtype != DType.F16 or buf.dtype != DType.F32:
        return None
    block = lowered.block_size
    forms: dict[int, Poly] = {}
    conj: dict[int, list[tuple[Poly, Poly]]] = {}
    for inst in ir.insts:
        o, op, a = inst.out, inst.op, inst.args
        if o is None:
            continue
        if op == "arg" and a[1] == "scalar" and o.dtype == DType.U32:
            forms[o.id] = {(f"${a[0]}",): 1}
        elif op == "const" and o.dtype == DType.U32:
            forms[o.id] = {(): int(a[0])} if int(a[0]) else {}
        elif op == "const" and o.dtype == DType.BOOL and a[0] is True:
            conj[o.id] = []
        elif op == "program_id":
            forms[o.id] = {(f"P{int(a[0])}",): 1}
        elif op == "thread_id":
            forms[o.id] = _padd({("P0",): block}, {("T",): 1}) if int(a[0]) == 0 else {(f"P{int(a[0])}",): 1}
        elif op == "tid":
            forms[o.id] = _padd({("T",): 1}, {(): int(a[0])} if int(a[0]) else {})
        elif op == "local_id":
            forms[o.id] = {("T",): 1} if int(a[0]) == 0 else {}
        elif op in ("add", "mul"):
            if a[0].id in forms and a[1].id in forms:
                fa, fb = forms[a[0].id], forms[a[1].id]
                forms[o.id] = _padd(fa, fb) if op == "add" else _pmul(fa, fb)
        elif op == "lt":
            if a[0].id in forms and a[1].id in forms:
                conj[o.id] = [(forms[a[0].id], forms[a[1].id])]
        elif op == "and":
            if a[0].id in conj and a[1].id in conj:
                conj[o.id] = conj[a[0].id] + conj[a[1].id]
    need = (a_base, b_base, a_stride, b_stride, k, off)
    if not all(x.id in forms for x in need) or mask.id not in conj:
        return None
    def ren(p: Poly) -> Poly:
        return p

    return DotGemmPlan(ir=ir, block=block, a_arg=arg_names[a_buf.id], b_arg=arg_names[b_buf.id],
                       c_arg=arg_names[buf.id], a_base=ren(forms[a_base.id]), b_base=ren(forms[b_base.id]),
                       a_stride=ren(forms[a_stride.id]), b_stride=ren(forms[b_stride.id]), k=ren(forms[k.id]),
                       c_off=ren(forms[off.id]), atoms=[(ren(l), ren(r)) for l, r in conj[mask.id]],
                       block_n=block if block in (128, 256) else 256)


def match_native(ir: IRModule, lowered: Any) -> Any:
    plan = _match_dot_gemm(ir, lowered)
    if plan is None:
        from .tiled import match_tiled

        plan = match_tiled(ir, lowered)
    if plan is None:
        from .mma_gemm import match_mma

        plan = match_mma(ir, lowered)
    return plan
