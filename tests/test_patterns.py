"""Native-pattern recognition (CPU): which IR maps onto the tcgen05 GEMM, with which strides."""

import numpy as np
import pytest

import goldens
from easy_as_b200.codegen.patterns import DotGemmPlan
from easy_as_b200.compiler import compile_ir
from examples.matmul_dot_f16 import matmul_dot_f16

import eas
from eas import mk


def _ck(M, N, K, batch, bn=256):
    a = np.zeros(1, np.float16)
    b = np.zeros(1, np.float16)
    c = np.zeros(1, np.float32)
    return matmul_dot_f16.compile(a, b, c, M, N, K, BLOCK_N=bn)


def _scal(M, N, K):
    return {"$M": M, "$N": N, "$K": K}


def test_dot_gemm_is_recognised():
    ck = _ck(8192, 8192, 8192, 1)
    assert isinstance(ck.plan.native, DotGemmPlan)
    assert ck.plan.native.block_n == 256


def test_c4_mapping():
    plan = _ck(8192, 8192, 8192, 1).plan.native
    m = plan.map_launch(_scal(8192, 8192, 8192), (32, 8192, 1), 0xFFFFFFFF)
    assert (m["M"], m["N"], m["K"], m["batch"]) == (8192, 8192, 8192, 1)
    assert (m["lda"], m["ldb"], m["b_kmajor"], m["ldc"]) == (8192, 8192, 0, 8192)


def test_c5_mapping_batched_runtime_k():
    plan = _ck(4096, 4096, 2088, 64).plan.native
    m = plan.map_launch(_scal(4096, 4096, 2088), (16, 4096, 64), 0xFFFFFFFF)
    assert (m["M"], m["N"], m["K"], m["batch"]) == (4096, 4096, 2088, 64)
    assert m["a_bs"] == 4096 * 2088 and m["b_bs"] == 2088 * 4096 and m["c_bs"] == 4096 * 4096
    assert m["lda"] == 2088 and m["ldb"] == 4096


def test_tails_clip_extents():
    plan = _ck(200, 300, 136, 3).plan.native
    m = plan.map_launch(_scal(200, 300, 136), (2, 200, 3), 0xFFFFFFFF)
    assert (m["M"], m["N"], m["batch"]) == (200, 300, 3)


def test_u32_wrap_is_rejected():
    # batch * (M*N) exceeds 2^32 for the C offsets: the generic kernel's wrapped semantics must be kept
    plan = _ck(8192, 8192, 64, 80).plan.native
    assert plan.map_launch(_scal(8192, 8192, 64), (32, 8192, 80), 0xFFFFFFFF) is None
    assert "wrap" in plan.last_reason


@eas.kernel
def gemm_nt(a, b, c, M, N, K, BLOCK: eas.constexpr):
    col = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    row = mk.program_id(1)
    inside = (row < M) & (col < N)
    mk.store(c, row * N + col, mk.dot(a, row * K, 1, b, col * K, 1, mk.where(inside, K, 0)), inside)


def test_k_major_b_is_recognised():
    ck = gemm_nt.compile(np.zeros(1, np.float16), np.zeros(1, np.float16), np.zeros(1, np.float32), 256, 512, 128,
                         BLOCK=128)
    m = ck.plan.native.map_launch(_scal(256, 512, 128), (4, 256, 1), 0xFFFFFFFF)
    assert m["b_kmajor"] == 1 and m["ldb"] == 128 and ck.plan.native.block_n == 128


@eas.kernel
def gemv_like_f32(a, x, y, M, K, BLOCK: eas.constexpr):
    row = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    mk.store(y, row, mk.dot(a, row * K, 1, x, 0, 1, K), row < M)


@pytest.mark.parametrize("cid", ["add_c1", "matmul_tiled_masked", "matmul_simdgroup", "t_gemv_dot", "t_tg_copy"])
def test_other_kernels_have_no_f16_gemm_plan(cid):
    """Other kernels may only carry the plans that prove their case per launch (tiled fp32 GEMM,
    simdgroup-MMA GEMM), never the f16 dot plan."""
    ck = compile_ir(goldens.ir_from_json(goldens.case(cid)["opt"]))
    assert getattr(ck.plan.native, "kind", None) in (None, "tiled_f32_ffma", "mma_f16_tcgen05")


def test_f32_dot_is_not_f16_gemm_pattern():
    ck = gemv_like_f32.compile(np.zeros(1, np.float32), np.zeros(1, np.float32), np.zeros(1, np.float32), 4, 4,
                               BLOCK=64)
    assert getattr(ck.plan.native, "kind", None) in (None, "tiled_f32_ffma")
