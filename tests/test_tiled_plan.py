"""The tiled fp32 GEMM proof (easy_as_b200/codegen/tiled.py) on CPU.

The reference's full-tile kernel (examples/matmul_tiled.py:134-230, IR from its
own front end) is proven to be one GEMM per launch, with the operand layout
read off the symbolic execution; kernels that differ in ways that change the
arithmetic or introduce races are declined.
"""

from __future__ import annotations

import dataclasses

import pytest

import goldens
from easy_as_b200.codegen.tiled import TiledGemmPlan, match_tiled
from easy_as_b200.compiler import compile_ir
from easy_as_b200.ir import Inst, IRModule


def _plan(cid):
    c = goldens.case(cid)
    ir = goldens.ir_from_json(c["opt"])
    return TiledGemmPlan(ir, c["block_size"]), c


def test_c3_kernel_is_one_2048_cube_gemm():
    plan, c = _plan("matmul_tiled_c3_full")
    d = plan.analyse({"M": 2048, "N": 2048}, (64, 64, 1), 64 * 256)
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"], d["batch"]) == (2048, 2048, 2048, 1)
    assert (d["kt"], d["ntile"], d["zero_init"]) == (32, 64, True)   # BK = 32 tiles, sum starts at 0.0f
    assert (d["a_sm"], d["b_sk"], d["c_sm"]) == (2048, 2048, 2048)
    assert (d["a_buf"], d["b_buf"], d["c_buf"]) == ("a", "b", "c")


def test_plan_is_attached_to_the_compiled_kernel():
    c = goldens.case("matmul_tiled_full")
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    assert ck.plan.native is not None and ck.plan.native.kind == "tiled_f32_ffma"


def test_small_full_tile_kernel_layout():
    plan, _ = _plan("matmul_tiled_full")
    d = plan.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256)
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"], d["a_sm"], d["b_sk"], d["c_sm"]) == (64, 128, 64, 64, 128, 128)


def test_grid_smaller_than_the_matrix_is_a_smaller_gemm():
    plan, _ = _plan("matmul_tiled_c3_full")
    d = plan.analyse({"M": 2048, "N": 2048}, (3, 2, 1), 3 * 256)
    assert d is not None and (d["M"], d["N"]) == (64, 96)


def test_ghost_threads_of_the_tiled_kernel_decline():
    """Ghost threads skip their threadgroup stores, so the tile would be incomplete."""
    plan, _ = _plan("matmul_tiled_full")
    assert plan.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256 - 3) is None
    assert "threadgroup store" in plan.last_reason
    assert plan.analyse({"M": 64, "N": 128}, (4, 2, 1), 0xFFFFFFFF) is not None  # explicit grid: all threads


def test_masked_tiled_kernel_is_a_zero_filled_gemm():
    plan, c = _plan("matmul_tiled_masked")
    d = plan.analyse({"M": 50, "N": 70, "PID_M_BASE": 0, "PID_N_BASE": 0}, (2, 4, 1), 0xFFFFFFFF)
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"], d["kt"]) == (50, 70, 64, 16)          # stores clipped to row < M, col < N
    assert (d["a_rows"], d["a_k"], d["b_cols"], d["b_k"]) == (50, 64, 70, 64)


def test_k_tail_mask_becomes_a_zero_filled_k_range():
    plan, c = _plan("t_matmul_tiled")                                       # K = 31 in tiles of 16
    d = plan.analyse({"M": 17, "N": 130}, (3, 2, 1), 0xFFFFFFFF)
    assert d is not None, plan.last_reason
    assert (d["K"], d["a_k"], d["b_k"], d["ntile"]) == (32, 31, 31, 2)


def test_pid_base_offsets_shift_the_bounds():
    plan, c = _plan("matmul_tiled_masked")
    # programs start at row group 1 and column group 1: rows 16.., columns 64.. of the matrices
    d = plan.analyse({"M": 50, "N": 150, "PID_M_BASE": 1, "PID_N_BASE": 1}, (1, 2, 1), 0xFFFFFFFF)
    assert d is not None, plan.last_reason
    assert (d["a0"], d["b0"], d["c0"]) == (16 * 64, 64, 16 * 150 + 64)
    assert (d["M"], d["N"], d["a_rows"], d["b_cols"]) == (32, 64, 32, 64)


def test_naive_fma_chain_with_ghost_threads_is_a_gemm():
    """examples/matmul.py: one fma chain per output, 1-D thread groups of 32 over W = 70 columns;
    the 26 ghost threads of the last group become the column bound."""
    plan, _ = _plan("matmul_naive")
    d = plan.analyse({"H": 40, "W": 70}, (3, 40, 1), 70)
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"], d["ntile"], d["zero_init"]) == (40, 70, 16, 1, False)
    assert (d["a_sm"], d["b_sk"], d["c_sm"]) == (16, 70, 70)


def test_operand_bound_on_the_other_coordinate():
    """t_matmul guards A and B with (row < M) & (col < N): harmless, since no output beyond it is kept."""
    plan, _ = _plan("t_matmul")
    assert plan.analyse({"M": 32, "N": 100}, (32, 2, 1), 0xFFFFFFFF) is not None


def _retarget_a_mask(ir: IRModule, extra: Inst, new_and: Inst) -> IRModule:
    """Insert ``extra`` and ``new_and`` before the first A load and make every A load use new_and."""
    a_id = next(i.out.id for i in ir.insts if i.op == "arg" and i.args[0] == "a")
    first = next(k for k, i in enumerate(ir.insts) if i.op == "load" and i.args[0].id == a_id)
    insts = list(ir.insts[:first]) + [extra, new_and]
    for i in ir.insts[first:]:
        if i.op == "load" and i.args[0].id == a_id:
            i = dataclasses.replace(i, args=(i.args[0], i.args[1], new_and.out))
        insts.append(i)
    return dataclasses.replace(ir, insts=tuple(insts))


def test_a_masked_by_column_inside_the_stored_range_declines():
    from easy_as_b200.ir import DType, ValueRef

    plan, c = _plan("t_matmul")
    ir = plan.ir
    col = next(i.args[0] for i in ir.insts if i.op == "lt" and i.args[1].id == 4)       # col < N
    mask = next(i.out for i in ir.insts if i.op == "and")
    c50 = ValueRef(9001, DType.U32)
    lt = ValueRef(9002, DType.BOOL)
    both = ValueRef(9003, DType.BOOL)
    ir2 = dataclasses.replace(ir, insts=(Inst("const", c50, (50,)),) + ir.insts)
    ir2 = _retarget_a_mask(ir2, Inst("lt", lt, (col, c50)), Inst("and", both, (mask, lt)))
    bad = TiledGemmPlan(ir2, c["block_size"])
    assert bad.analyse({"M": 32, "N": 100}, (32, 2, 1), 0xFFFFFFFF) is None
    assert "other operand" in bad.last_reason


def test_triangular_mask_declines():
    from easy_as_b200.ir import DType, ValueRef

    plan, c = _plan("t_matmul")
    ir = plan.ir
    row = next(i.args[0] for i in ir.insts if i.op == "lt" and i.args[1].id == 3)       # row < M
    col = next(i.args[0] for i in ir.insts if i.op == "lt" and i.args[1].id == 4)
    mask = next(i.out for i in ir.insts if i.op == "and")
    lt = ValueRef(9002, DType.BOOL)
    both = ValueRef(9003, DType.BOOL)
    ir2 = _retarget_a_mask(ir, Inst("lt", lt, (col, row)), Inst("and", both, (mask, lt)))
    bad = TiledGemmPlan(ir2, c["block_size"])
    assert bad.analyse({"M": 32, "N": 100}, (32, 2, 1), 0xFFFFFFFF) is None


def _without(ir: IRModule, op: str) -> IRModule:
    return dataclasses.replace(ir, insts=tuple(i for i in ir.insts if i.op != op))


def test_missing_barriers_are_a_race_and_decline():
    plan, c = _plan("matmul_tiled_full")
    racy = TiledGemmPlan(_without(plan.ir, "barrier"), c["block_size"])
    assert racy.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256) is None
    assert "barrier" in racy.last_reason


def test_a_changed_accumulation_declines():
    """Replace one running-sum add by a mul: the stored value is no longer a fold of dots."""
    plan, c = _plan("matmul_tiled_full")
    insts = list(plan.ir.insts)
    k = max(i for i, x in enumerate(insts) if x.op == "add" and x.out.dtype.name == "F32")
    insts[k] = dataclasses.replace(insts[k], op="mul")
    bad = TiledGemmPlan(dataclasses.replace(plan.ir, insts=tuple(insts)), c["block_size"])
    assert bad.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256) is None


def test_index_wrap_declines():
    plan, _ = _plan("matmul_tiled_c3_full")
    # N so large that row * N overflows u32 for the last row group
    assert plan.analyse({"M": 2048, "N": 1 << 22}, (64, 64, 1), 64 * 256) is None


def test_static_filter_rejects_spmd_and_dotless_kernels():
    for cid in ("add_c1", "t_tg_copy"):
        c = goldens.case(cid)
        ck = compile_ir(goldens.ir_from_json(c["opt"]))
        assert match_tiled(ck.ir, ck.plan) is None


def test_proof_results_are_cached_on_disk(tmp_path, monkeypatch):
    monkeypatch.setenv("EAS_CACHE_DIR", str(tmp_path))
    c = goldens.case("matmul_tiled_full")
    ir = goldens.ir_from_json(c["opt"])
    first = TiledGemmPlan(ir, c["block_size"]).analyse({"M": 64, "N": 128}, (4, 2, 1), 0xFFFFFFFF)
    files = list((tmp_path / "plans").glob("*.json"))
    assert len(files) == 1
    again = TiledGemmPlan(ir, c["block_size"]).analyse({"M": 64, "N": 128}, (4, 2, 1), 0xFFFFFFFF)
    assert again == first
    # declines are cached too, with their reason
    bad = TiledGemmPlan(ir, c["block_size"])
    assert bad.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256 - 3) is None
    reason = bad.last_reason
    bad2 = TiledGemmPlan(ir, c["block_size"])
    assert bad2.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256 - 3) is None and bad2.last_reason == reason
    monkeypatch.setenv("EAS_PLAN_CACHE", "0")
    TiledGemmPlan(ir, c["block_size"]).analyse({"M": 64, "N": 256}, (8, 2, 1), 0xFFFFFFFF)
    assert len(list((tmp_path / "plans").glob("*.json"))) == 2


def test_program_id_sub_range_is_the_shifted_gemm():
    """Programs 32..63 along y of the C3 launch: rows 1024..2047 of the same GEMM."""
    plan, _ = _plan("matmul_tiled_c3_full")
    d = plan.analyse({"M": 2048, "N": 2048}, (64, 32, 1), 0xFFFFFFFF, pid_base=(0, 32, 0))
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"]) == (1024, 2048, 2048)
    assert (d["a0"], d["b0"], d["c0"]) == (1024 * 2048, 0, 1024 * 2048)


def test_own_tiled_variants_are_proven():
    """Kernels of another shape than the reference's (tests/tiled_variants.py) are proven too."""
    import numpy as np

    from tiled_variants import VARIANTS, grid, tile_mm

    M, N, K = 70, 150, 48
    for tm, tn, tk, nt, pad in VARIANTS:
        kk = -(-K // tk) * tk if K % tk else K
        ck = tile_mm.compile(np.zeros(M * kk, np.float32), np.zeros(kk * N, np.float32), np.zeros(M * N, np.float32),
                             M, N, K=K, TM=tm, TN=tn, TK=tk, NT=nt, PAD=pad)
        plan = ck.plan.native
        assert plan is not None and plan.kind == "tiled_f32_ffma"
        d = plan.analyse({"M": M, "N": N}, grid(M, N, tm, tn), 0xFFFFFFFF)
        assert d is not None, (tm, tn, tk, nt, pad, plan.last_reason)
        assert (d["M"], d["N"], d["a_k"], d["kt"]) == (M, N, K, tk)


def test_batched_variant_maps_the_z_axis_to_the_batch():
    import numpy as np

    from tiled_variants import tile_mm_batched

    M, N, K = 70, 150, 64
    ck = tile_mm_batched.compile(np.zeros(1, np.float32), np.zeros(1, np.float32), np.zeros(1, np.float32), M, N,
                                 K=K, TM=32, TN=32, TK=16, NT=128)
    d = ck.plan.native.analyse({"M": M, "N": N}, (5, 3, 5), 0xFFFFFFFF)
    assert d is not None, ck.plan.native.last_reason
    assert (d["batch"], d["a_bs"], d["b_bs"], d["c_bs"]) == (5, M * K, K * N, M * N)


def test_fp32_matmul_mode_knob(monkeypatch):
    from easy_as_b200.codegen.tiled import fp32_mode

    monkeypatch.delenv("EAS_FP32_MATMUL", raising=False)
    assert fp32_mode() == "exact"
    monkeypatch.setenv("EAS_FP32_MATMUL", "3xTF32")
    assert fp32_mode() == "3xtf32"
    monkeypatch.setenv("EAS_FP32_MATMUL", "tf32")
    with pytest.raises(ValueError):
        fp32_mode()
