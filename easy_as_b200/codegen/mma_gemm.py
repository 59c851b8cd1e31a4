"""Prove that a simdgroup-MMA kernel is an f16 GEMM with f32 accumulation, and run it on tcgen05.

Target: the reference's ``matmul_simdgroup_mma_kernel`` (easy_as
``examples/matmul_simdgroup.py:29-127``): threads copy f32 A and B tiles into threadgroup memory
cast to f16, each simdgroup (warp) multiplies 8x8 tiles with ``mk.mma`` into an f32 fragment,
stores the fragment to threadgroup memory, and threads copy it to C.  The reference's
accumulation order inside ``simdgroup_multiply_accumulate`` is unspecified (Apple's matrix unit;
the example checks 5e-3 against an fp16-cast reference), so what must be proven is *which*
products every output sums: f16(A[m][k]) * f16(B[k][n]) for each k of the K range exactly once,
in f32.

The symbolic execution of :mod:`.tiled` (linear program-id forms, masks as rectangle atoms,
race-free threadgroup memory by barrier phases) is extended with

* ``cast`` f32 -> f16 of a global load (kept as a flag on the threadgroup slot it is stored to);
* ``mma``: per warp (its operand bases must be the same in all 32 lanes), an 8x8x8 step whose
  A slots are ``a_base + r*a_stride + kk`` and B slots ``b_base + kk*b_stride + c``; a fragment
  is the list of its steps;
* ``mma_store``: fragment element (r, c) of warp w to slot ``base_w + r*stride + c``; a later
  load of such a slot yields that element.

A global store of fragment elements becomes, per thread, the K products of its element sorted by
A address, i.e. one dot per output, and the rest of the proof (one GEMM per launch, rectangle
masks, program-id shifts) is the tiled one.  The launch writes A and B once as zero-filled f16
(``eas_cast_f32_f16_2d``, the same rounding as the kernel's cast) and runs ``eas_gemm_f16``
(tcgen05, f32 accumulation).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np

from ..ir import DType, IRModule, Inst, ValueRef
from .tiled import FDot, FLoad, ProvenGemmPlan, Side, _affine_k, _Exec, _need, _Smem, _uniform_rhs


@dataclass(frozen=True, eq=False)
class FCast16:
    x: FLoad


@dataclass(frozen=True, eq=False)
class FFrag:
    steps: tuple[tuple[dict, dict], ...]      # per mma: (A operand, B operand) slot data per warp


@dataclass(frozen=True, eq=False)
class FFragElem:
    frag: FFrag
    w: np.ndarray      # (NT,) warp of the element
    r: np.ndarray
    c: np.ndarray


class _MmaSmem(_Smem):
    def __init__(self, n: int):
        super().__init__(n)
        self.cast = np.zeros(n, np.bool_)          # slot holds f16(load)
        self.fidx = np.full(n, -1, np.int64)       # fragment element: index into _MmaExec.frags
        self.fw = np.zeros(n, np.int64)
        self.fr = np.zeros(n, np.int64)
        self.fc = np.zeros(n, np.int64)


class _MmaExec(_Exec):
    def __init__(self, *a: Any, **k: Any):
        super().__init__(*a, **k)
        self.frags: list[FFrag] = []
        self.warps = self.nt // 32
        _need(self.nt % 32 == 0, "thread group is not whole warps")

    def op_alloc_tg(self, inst: Inst) -> None:
        _need(inst.out.dtype in (DType.F32, DType.F16), "threadgroup memory of another type")
        self.smem[inst.out.id] = _MmaSmem(int(inst.args[0]))
        self.vals[inst.out.id] = ("smem", inst.out.id)

    def op_cast(self, inst: Inst) -> None:
        x, dst = inst.args
        v = self.vals[x.id]
        _need(x.dtype == DType.F32 and inst.out.dtype == DType.F16 and isinstance(v, FLoad),
              "cast other than f32 load -> f16")
        self.vals[inst.out.id] = FCast16(v)

    def op_load(self, inst: Inst) -> None:
        buf, off, mask = inst.args
        kind, ident = self._buffer(buf)
        if kind == "gbuf":
            super().op_load(inst)
            return
        m = self.plain(mask)
        _need(bool(m.all()), "masked threadgroup load")
        sm = self.smem[ident]
        slots = self.concrete(off).astype(np.int64)
        _need(bool((slots < len(sm.buf)).all()), "threadgroup load out of range")
        _need(bool((sm.fidx[slots] >= 0).all()), "threadgroup load of something other than an mma result")
        _need(bool((sm.wphase[slots] < self.phase).all()), "threadgroup load of a slot written since the last barrier")
        sm.rphase[slots] = self.phase
        f = sm.fidx[slots]
        _need(bool((f == f[0]).all()), "threadgroup loads from different mma fragments")
        self.vals[inst.out.id] = FFragElem(self.frags[int(f[0])], sm.fw[slots], sm.fr[slots], sm.fc[slots])

    def op_mma_zero(self, inst: Inst) -> None:
        self.vals[inst.out.id] = FFrag(())

    def _warp_uniform(self, ref: ValueRef, what: str) -> np.ndarray:
        v = self.concrete(ref).astype(np.int64).reshape(self.warps, 32)
        _need(bool((v == v[:, :1]).all()), f"{what} differs between the lanes of a warp")
        return v[:, 0]

    def _operand(self, buf: ValueRef, base: ValueRef, stride: ValueRef) -> dict:
        kind, ident = self._buffer(buf)
        _need(kind == "smem", "mma operand outside threadgroup memory")
        sm = self.smem[ident]
        b = self._warp_uniform(base, "mma base")
        st = self.scalar_const(stride)
        i8 = np.arange(8, dtype=np.int64)
        # A[w][r][kk] at base + r*stride + kk;  B[w][kk][c] at base + kk*stride + c
        slots = b[:, None, None] + i8[None, :, None] * st + i8[None, None, :]
        _need(bool(((slots >= 0) & (slots < len(sm.buf))).all()), "mma reads outside threadgroup memory")
        _need(bool((sm.wphase[slots] >= 0).all()), "mma reads an unwritten slot")
        _need(bool((sm.wphase[slots] < self.phase).all()), "mma reads a slot written since the last barrier")
        _need(bool((sm.fidx[slots] < 0).all()), "mma operand holds an mma result")
        codes = sm.buf[slots]
        _need(bool((codes == codes.flat[0]).all()), "mma operand loaded from different buffers")
        _need(bool(sm.cast[slots].all()), "mma operand not an f16 cast of an f32 load")
        sm.rphase[slots.ravel()] = self.phase
        return {"buf": self.name_of(int(codes.flat[0])), "lin": sm.lin[:, slots], "conc": sm.conc[slots],
                "rec": sm.rec[slots], "writer": sm.writer[slots]}

    def op_mma(self, inst: Inst) -> None:
        a_buf, a_base, a_stride, b_buf, b_base, b_stride, acc = inst.args
        prev = self.vals[acc.id]
        _need(isinstance(prev, FFrag), "mma accumulator is not a fragment")
        step = (self._operand(a_buf, a_base, a_stride), self._operand(b_buf, b_base, b_stride))
        self.vals[inst.out.id] = FFrag(prev.steps + (step,))

    def op_mma_store(self, inst: Inst) -> None:
        buf, base, stride, frag = inst.args
        f = self.vals[frag.id]
        _need(isinstance(f, FFrag) and f.steps, "mma_store of an empty fragment")
        kind, ident = self._buffer(buf)
        _need(kind == "smem", "mma_store outside threadgroup memory")
        sm = self.smem[ident]
        b = self._warp_uniform(base, "mma_store base")
        st = self.scalar_const(stride)
        i8 = np.arange(8, dtype=np.int64)
        slots = b[:, None, None] + i8[None, :, None] * st + i8[None, None, :]      # (W, 8, 8)
        _need(bool(((slots >= 0) & (slots < len(sm.buf))).all()), "mma_store outside threadgroup memory")
        flat = slots.ravel()
        _need(len(np.unique(flat)) == len(flat), "mma_store elements overlap")
        _need(bool((sm.wphase[flat] != self.phase).all()), "slot written twice between barriers")
        _need(bool((sm.rphase[flat] != self.phase).all()), "slot written after a read between barriers")
        self.frags.append(f)
        ww, rr, cc = np.meshgrid(np.arange(self.warps), i8, i8, indexing="ij")
        sm.fidx[flat] = len(self.frags) - 1
        sm.fw[flat], sm.fr[flat], sm.fc[flat] = ww.ravel(), rr.ravel(), cc.ravel()
        sm.buf[flat] = -1
        sm.wphase[flat] = self.phase

    def _slot_load(self, v: Any) -> tuple[FLoad, Any]:
        if isinstance(v, FCast16):
            return v.x, True
        return super()._slot_load(v)[0], False

    def _slot_written(self, sm: _Smem, slots: np.ndarray, extra: Any) -> None:
        sm.cast[slots] = bool(extra)
        sm.fidx[slots] = -1

    def run(self) -> None:
        super().run()
        self.stores = [(b, off, self._as_dot(v), m) if isinstance(v, FFragElem) else (b, off, v, m)
                       for b, off, v, m in self.stores]

    def _as_dot(self, e: FFragElem) -> FDot:
        """The products of each thread's fragment element, sorted by A address, as one dot."""
        parts_a, parts_b = [], []
        for a_op, b_op in e.frag.steps:
            # A[w][r][kk] and B[w][kk][c] of each thread's element (w, r, c): 8 products per step
            parts_a.append({"lin": a_op["lin"][:, e.w, e.r, :], **{k: a_op[k][e.w, e.r, :]
                                                                   for k in ("conc", "rec", "writer")}})
            parts_b.append({"lin": np.transpose(b_op["lin"][:, e.w, :, e.c], (1, 0, 2)),
                            **{k: b_op[k][e.w, :, e.c] for k in ("conc", "rec", "writer")}})
        bufs = {(a["buf"], b["buf"]) for a, b in e.frag.steps}
        _need(len(bufs) == 1, "mma steps read different buffers")
        a_name, b_name = bufs.pop()
        cat = {}
        for side, parts in (("a", parts_a), ("b", parts_b)):
            cat[side] = {"lin": np.concatenate([p["lin"] for p in parts], axis=2),       # (4, NT, Kp)
                         "conc": np.concatenate([p["conc"] for p in parts], axis=1),     # (NT, Kp)
                         "rec": np.concatenate([p["rec"] for p in parts], axis=1),
                         "writer": np.concatenate([p["writer"] for p in parts], axis=1)}
        order = np.argsort(cat["a"]["lin"][0], axis=1, kind="stable")
        sides = []
        for side, name in (("a", a_name), ("b", b_name)):
            d = cat[side]
            lin = np.take_along_axis(d["lin"], order[None, :, :], axis=2)
            conc = np.take_along_axis(d["conc"], order, axis=1)
            rec = np.take_along_axis(d["rec"], order, axis=1)
            writer = np.take_along_axis(d["writer"], order, axis=1)
            base, step = _affine_k(lin, f"mma {side} addresses")
            sides.append(Side(name, base, step, conc, self._atoms(rec, writer)))
        return FDot(sides[0], sides[1], order.shape[1])

    def _atoms(self, rec: np.ndarray, writer: np.ndarray) -> tuple:
        recs = np.unique(rec)
        na = len(self.records[int(recs[0])])
        _need(all(len(self.records[int(r)]) == na for r in recs), "products loaded under different mask shapes")
        atoms = []
        for a in range(na):
            lhs = np.zeros((4,) + rec.shape, np.uint64)
            rhs = np.zeros((4,) + rec.shape, np.uint64)
            for r in recs:
                pos = rec == r
                l_r, r_r = self.records[int(r)][a]
                lhs[:, pos] = l_r[:, writer[pos]]
                rhs[:, pos] = r_r[:, writer[pos]]
            l0, ls = _affine_k(lhs, "mask bound")
            atoms.append((l0, ls, _uniform_rhs(rhs, "mask")))
        return tuple(atoms)


_OPS = {"arg", "const", "alloc_tg", "program_id", "thread_id", "tid", "local_id", "lane_id", "sg_id", "add", "mul",
        "floordiv", "mod", "lt", "and", "or", "not", "where", "barrier", "load", "store", "cast", "mma_zero", "mma",
        "mma_store"}


class MmaGemmPlan(ProvenGemmPlan):
    """tcgen05 launch for simdgroup-MMA kernels proven to be f16 GEMMs (module docstring)."""

    kind = "mma_f16_tcgen05"
    executor = _MmaExec
    allow_ghosts = False

    def _launch(self, rt: Any, d: dict[str, Any], pa: int, pb: int, pc: int, device: int, stream: int) -> bool:
        from ..runtime import cuda_ext

        M, N, K, batch = d["M"], d["N"], d["K"], d["batch"]
        n_pad = -(-N // 8) * 8
        sa = rt.scratch(device, stream, "mma_a16", 2 * batch * M * K)
        sb = rt.scratch(device, stream, "mma_b16", 2 * batch * K * n_pad)
        if sa is None or sb is None:
            self.last_reason = "f16 staging buffers cannot be allocated during graph capture"
            return False
        (a16, _keep_a), (b16, _keep_b) = sa, sb          # owners stay alive until the launches are enqueued
        lib = rt.lib()
        cuda_ext.check(lib.eas_cast_f32_f16_2d(pa + 4 * d["a0"], a16, M, K, d["a_sm"], K, d["a_rows"], d["a_k"], batch,
                                               d["a_bs"], M * K, stream), "cast A to f16")
        cuda_ext.check(lib.eas_cast_f32_f16_2d(pb + 4 * d["b0"], b16, K, n_pad, d["b_sk"], n_pad, d["b_k"],
                                               d["b_cols"], batch, d["b_bs"], K * n_pad, stream), "cast B to f16")
        rc = lib.eas_gemm_f16(a16, b16, pc + 4 * d["c0"], M, N, K, batch, K, M * K, n_pad, K * n_pad, 0,
                              d["c_sm"] if M > 1 else N, d["c_bs"], 256 if M > 128 else 128, stream)
        if rc == cuda_ext.EAS_ERR_VALUE:
            self.last_reason = cuda_ext.last_error()
            return False
        cuda_ext.check(rc, "gemm_f16 (tcgen05) for an mma kernel")
        rt.launch_count += 3
        rt.native_launches += 1
        return True


def match_mma(ir: IRModule, lowered: Any) -> MmaGemmPlan | None:
    """Cheap static filter; the proof runs per launch."""
    if lowered.mode != "thread":
        return None
    if any(i.op not in _OPS for i in ir.insts):
        return None
    if not any(i.op == "mma" for i in ir.insts):
        return None
    return MmaGemmPlan(ir, lowered.block_size)
