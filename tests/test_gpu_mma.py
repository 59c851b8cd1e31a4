"""GPU: the reference's simdgroup-MMA matmul (IR from its front end) proven to be an f16 GEMM runs on
the tcgen05 kernel over f16-cast operands.

The reference leaves the accumulation order of ``simdgroup_multiply_accumulate`` unspecified and
its example checks rtol = atol = 5e-3 against an fp16-cast product
(examples/matmul_simdgroup.py:218-227).  Here the native result is held to that bar against the
generated kernel and the CPU oracle, and to 1e-5 normwise against float64 on the same f16-rounded
inputs (exact f16 products, f32 accumulation)."""

from __future__ import annotations

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from oracle.interp import execute

pytestmark = pytest.mark.gpu


def _f16_ref(a, b, M, N, K):
    a16 = a.reshape(M, K).astype(np.float16).astype(np.float64)
    b16 = b.reshape(K, N).astype(np.float16).astype(np.float64)
    return a16 @ b16


@pytest.mark.parametrize("cid,M,N", [("matmul_simdgroup", 40, 36), ("matmul_simdgroup", 100, 70),
                                     ("matmul_simdgroup_512", 512, 512), ("matmul_simdgroup_512", 300, 200)])
def test_native_mma_gemm(cuda_rt, monkeypatch, cid, M, N):
    c = goldens.case(cid)
    ir = goldens.ir_from_json(c["opt"])
    ck = compile_ir(ir)
    assert ck.plan.native is not None and ck.plan.native.kind == "mma_f16_tcgen05"
    K = c["meta"]["K"]
    meta = c["meta"]
    grid = (-(-N // meta["BN"]), -(-M // meta["BM"]), 1)
    rng = np.random.default_rng(M * N)
    a = rng.standard_normal(M * K).astype(np.float32)
    b = rng.standard_normal(K * N).astype(np.float32)
    native = np.full(M * N, np.nan, np.float32)
    before = cuda_rt.native_launches
    cuda_rt.run(ck, {"a": a, "b": b, "c": native, "M": M, "N": N}, meta, sync=True, grid=grid)
    assert cuda_rt.native_launches == before + 1, ck.plan.native.last_reason
    ref = _f16_ref(a, b, M, N, K)
    err = np.abs(native.reshape(M, N) - ref).max() / np.abs(ref).max()
    assert err <= 1e-5, err
    monkeypatch.setenv("EAS_DISABLE_NATIVE", "1")
    generic = np.full(M * N, np.nan, np.float32)
    cuda_rt.run(ck, {"a": a, "b": b, "c": generic, "M": M, "N": N}, meta, sync=True, grid=grid)
    np.testing.assert_allclose(native, generic, rtol=5e-3, atol=5e-3)
    if M * N <= 100 * 70:
        cpu = np.zeros(M * N, np.float32)
        execute(ir, {"a": a, "b": b, "c": cpu, "M": M, "N": N}, grid=grid)
        np.testing.assert_allclose(native, cpu, rtol=5e-3, atol=5e-3)
