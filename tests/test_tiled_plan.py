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
from easy_as_b200.ir import IRModule


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


def test_ghost_threads_decline():
    plan, _ = _plan("matmul_tiled_full")
    assert plan.analyse({"M": 64, "N": 128}, (4, 2, 1), 4 * 256 - 3) is None
    assert "ghost" in plan.last_reason
    assert plan.analyse({"M": 64, "N": 128}, (4, 2, 1), 0xFFFFFFFF) is not None  # explicit grid: all threads


@pytest.mark.parametrize("cid", ["matmul_tiled_masked", "t_matmul_tiled"])
def test_masked_kernels_decline(cid):
    c = goldens.case(cid)
    plan = TiledGemmPlan(goldens.ir_from_json(c["opt"]), c["block_size"])
    scal = {n: v for n, v in zip(c["arg_names"], c["args"]) if not isinstance(v, dict)}
    g = c["launch"]["grid"]
    assert plan.analyse(scal, tuple(g), g[0] * c["block_size"]) is None


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
