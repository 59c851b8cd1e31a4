"""Re-rolling of Python-unrolled loops (easy_as_b200/codegen/reroll.py) on CPU.

Every run found in the reference kernels' IR is expanded back from its
operand forms and compared, instruction by instruction, with the original
unrolled IR: the loop the emitter prints then performs exactly the unrolled
operations in the same order.  The printed sources compile with NVRTC for
sm_100a.  Bit-for-bit results on the device are covered by the GPU parity
tests, which run the re-rolled sources against the CPU oracle.
"""

from __future__ import annotations

import ctypes

import pytest

import goldens
from easy_as_b200.codegen.cuda import _Emitter, ir_to_cuda
from easy_as_b200.codegen.reroll import find_runs
from easy_as_b200.ir import DType, Inst, ValueRef
from easy_as_b200.runtime import cuda_ext

CASES = goldens.cases() + goldens.big_cases()
IDS = [c["id"] for c in CASES]


def _u32_consts(insts):
    return {i.out.id: int(i.args[0]) for i in insts if i.op == "const" and i.out.dtype == DType.U32
            and not isinstance(i.args[0], bool)}


def _check_run(insts, run) -> None:
    u32 = _u32_consts(insts)
    outs = [[None if insts[k].out is None else insts[k].out.id for k in b] for b in run.blocks]
    for r, block in enumerate(run.blocks):
        for j, k in enumerate(block):
            inst, base = insts[k], insts[run.first[j]]
            assert inst.op == base.op and len(inst.args) == len(base.args)
            assert (inst.out is None) == (base.out is None)
            if inst.out is not None:
                assert (inst.out.dtype, inst.out.lanes) == (base.out.dtype, base.out.lanes)
            for a, f in zip(inst.args, run.forms[j]):
                kind = f[0]
                if kind == "lit":
                    assert not isinstance(a, ValueRef)  # literal values compared below
                elif kind == "local":
                    assert a.id == outs[r][f[1]]
                elif kind == "carry":
                    assert a.id == (f[2] if r == 0 else outs[r - 1][f[1]])
                elif kind == "inv":
                    assert a.id == f[1]
                elif kind == "affine":
                    assert u32[a.id] == (f[1] + r * f[2]) % (1 << 32)
                else:
                    raise AssertionError(kind)
            lits = [a for a in inst.args if not isinstance(a, ValueRef)]
            assert lits == [a for a in base.args if not isinstance(a, ValueRef)]
    span = run.ir_span
    for k, inst in enumerate(insts):
        if k in span:
            continue
        for a in inst.args:
            if not isinstance(a, ValueRef):
                continue
            for r, block in enumerate(run.blocks):
                if a.id in outs[r]:
                    assert r == run.count - 1, "a value of an inner block is read after the run"
                    assert outs[r].index(a.id) in run.escapes


@pytest.mark.parametrize("c", CASES, ids=IDS)
def test_runs_expand_to_the_unrolled_ir(c):
    ir = goldens.ir_from_json(c["opt"])
    groups = _Emitter(ir)._dot_groups()
    keep = tuple(frozenset(m) for m in groups.values() if m)
    runs = find_runs(ir.insts, keep_together=keep)
    covered: set[int] = set()
    for run in runs:
        assert run.count >= 3
        assert not (covered & run.ir_span)
        covered |= run.ir_span
        _check_run(ir.insts, run)
        for g in keep:
            assert len({next((r for r, b in enumerate(run.blocks) if k in b), None) for k in g}) == 1


def test_bench_scale_tiled_kernel_becomes_one_loop():
    c = goldens.case("matmul_tiled_c3_full")
    ir = goldens.ir_from_json(c["opt"])
    runs = find_runs(ir.insts)
    assert max(r.count for r in runs) >= 60  # 64 K tiles of 32
    src = ir_to_cuda(ir).src
    assert src.count("\n") < 600 and "for (uint32_t eas_r" in src


def test_reroll_can_be_switched_off(monkeypatch):
    ir = goldens.ir_from_json(goldens.case("matmul_naive")["opt"])
    assert "eas_r" in ir_to_cuda(ir).src
    monkeypatch.setenv("EAS_REROLL", "0")
    assert "eas_r" not in ir_to_cuda(ir).src


def _v(i, dt=DType.U32):
    return ValueRef(i, dt)


def _chain(n_blocks, offsets, read_inner_after=False):
    """x[off_r] += 1 for r in blocks, as straight-line IR (load, add, store per block)."""
    insts = [Inst("arg", _v(0, DType.F32), ("x",)), Inst("const", _v(1, DType.BOOL), (True,)),
             Inst("const", _v(2, DType.F32), (1.0,))]
    nid = 3
    vals = []
    for r in range(n_blocks):
        insts.append(Inst("const", _v(nid), (offsets[r],)))
        off = nid
        insts.append(Inst("load", _v(nid + 1, DType.F32), (_v(0, DType.F32), _v(off), _v(1, DType.BOOL))))
        insts.append(Inst("add", _v(nid + 2, DType.F32), (_v(nid + 1, DType.F32), _v(2, DType.F32))))
        insts.append(Inst("store", None, (_v(0, DType.F32), _v(off), _v(nid + 2, DType.F32), _v(1, DType.BOOL))))
        vals.append(nid + 2)
        nid += 3
    if read_inner_after:
        insts.append(Inst("store", None, (_v(0, DType.F32), _v(3), _v(vals[1], DType.F32), _v(1, DType.BOOL))))
    return insts


def test_affine_offsets_roll_and_irregular_ones_do_not():
    runs = find_runs(tuple(_chain(12, [4 * r + 8 for r in range(12)])), min_saved=3)
    assert len(runs) == 1 and runs[0].count == 12
    assert ("affine", 8, 4) in runs[0].forms[0]
    irregular = [0, 1, 3, 7, 15, 31, 63, 127, 255, 511, 1023, 2047]
    assert find_runs(tuple(_chain(12, irregular)), min_saved=3) == []


def test_inner_block_value_read_after_the_run_blocks_rolling():
    runs = find_runs(tuple(_chain(12, [4 * r for r in range(12)], read_inner_after=True)), min_saved=3)
    for run in runs:
        _check_run(tuple(_chain(12, [4 * r for r in range(12)], read_inner_after=True)), run)


@pytest.mark.parametrize("cid", ["matmul_naive", "matmul_tiled_masked", "t_many_dot", "matmul_tiled_c3_full"])
def test_rerolled_sources_compile(cid):
    lo = ir_to_cuda(goldens.ir_from_json(goldens.case(cid)["opt"]))
    lib = cuda_ext.load()
    img, size = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.eas_compile(lo.src.encode(), (lo.kernel_name + ".cu").encode(), None, 0, ctypes.byref(img),
                         ctypes.byref(size))
    if rc == cuda_ext.EAS_ERR_UNAVAILABLE:
        pytest.skip("NVRTC not loadable here")
    assert rc == 0, cuda_ext.last_error()
    lib.eas_free_host(img)


@pytest.mark.parametrize("name", ["colsum", "rows_scale"])
def test_spmd_loops_are_rerolled_and_compile(name, monkeypatch):
    import numpy as np

    import spmd_loops

    k = getattr(spmd_loops, name)
    x = np.zeros(64 * 1000, np.float32)
    y = np.zeros(64 * 1000, np.float32)
    src = k.compile(x, y, 1000, W=64, BLOCK=256).src
    assert "for (uint32_t eas_r" in src and src.count("\n") < 400
    for run in find_runs(k.compile(x, y, 1000, W=64, BLOCK=256).ir.insts):
        _check_run(k.compile(x, y, 1000, W=64, BLOCK=256).ir.insts, run)
    lib = cuda_ext.load()
    img, size = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.eas_compile(src.encode(), b"k.cu", None, 0, ctypes.byref(img), ctypes.byref(size))
    if rc == cuda_ext.EAS_ERR_UNAVAILABLE:
        pytest.skip("NVRTC not loadable here")
    assert rc == 0, cuda_ext.last_error()
    lib.eas_free_host(img)
    from easy_as_b200.compiler import compile_ir

    monkeypatch.setenv("EAS_REROLL", "0")      # the kernel's compile cache is bypassed: lower the IR again
    assert "eas_r" not in compile_ir(k.compile(x, y, 1000, W=64, BLOCK=256).ir).src
