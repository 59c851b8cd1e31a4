"""The simdgroup-MMA GEMM proof (easy_as_b200/codegen/mma_gemm.py) on CPU, on the reference's
matmul_simdgroup_mma_kernel IR (examples/matmul_simdgroup.py:29-127, from its front end)."""

from __future__ import annotations

import dataclasses

import goldens
from easy_as_b200.codegen.mma_gemm import MmaGemmPlan
from easy_as_b200.compiler import compile_ir


def _plan(cid):
    c = goldens.case(cid)
    return MmaGemmPlan(goldens.ir_from_json(c["opt"]), c["block_size"]), c


def test_golden_kernel_is_an_f16_gemm():
    plan, c = _plan("matmul_simdgroup")                       # 40 x 36 x 32, BM = BN = BK = 16
    d = plan.analyse({"M": 40, "N": 36}, tuple(c["launch"]["grid"]), 0xFFFFFFFF)
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"], d["batch"]) == (40, 36, 32, 1)
    assert (d["a_sm"], d["b_sk"], d["c_sm"]) == (32, 36, 36)
    assert (d["a_rows"], d["a_k"], d["b_cols"], d["b_k"]) == (40, 32, 36, 32)


def test_example_default_run_is_an_f16_gemm():
    plan, c = _plan("matmul_simdgroup_512")                   # 512^3, BM=16 BN=32 BK=8
    d = plan.analyse({"M": 512, "N": 512}, tuple(c["launch"]["grid"]), 0xFFFFFFFF)
    assert d is not None, plan.last_reason
    assert (d["M"], d["N"], d["K"]) == (512, 512, 512)


def test_plan_is_attached():
    ck = compile_ir(goldens.ir_from_json(goldens.case("matmul_simdgroup")["opt"]))
    assert ck.plan.native is not None and ck.plan.native.kind == "mma_f16_tcgen05"


def test_missing_barrier_declines():
    plan, c = _plan("matmul_simdgroup")
    ir = dataclasses.replace(plan.ir, insts=tuple(i for i in plan.ir.insts if i.op != "barrier"))
    bad = MmaGemmPlan(ir, c["block_size"])
    assert bad.analyse({"M": 40, "N": 36}, tuple(c["launch"]["grid"]), 0xFFFFFFFF) is None


def test_repeated_k_step_declines():
    """Feeding the second mma the first one's tiles sums k = 0..7 twice and never 8..15."""
    plan, c = _plan("matmul_simdgroup")
    insts = list(plan.ir.insts)
    k = next(i for i, x in enumerate(insts) if x.op == "mma")
    nxt = next(i for i, x in enumerate(insts) if i > k and x.op == "mma")
    insts[nxt] = dataclasses.replace(insts[nxt], args=insts[k].args[:6] + insts[nxt].args[6:])
    bad = MmaGemmPlan(dataclasses.replace(plan.ir, insts=tuple(insts)), c["block_size"])
    assert bad.analyse({"M": 40, "N": 36}, tuple(c["launch"]["grid"]), 0xFFFFFFFF) is None
    assert "affine" in bad.last_reason
