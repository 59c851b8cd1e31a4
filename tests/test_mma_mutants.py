"""CPU: the simdgroup-MMA GEMM proof on near-miss variants of a DSL simdgroup-MMA matmul
(tests/mma_mutants.py): the unchanged kernel is proven an f16 GEMM, mutants that are not GEMMs
are declined.  Accepted mutants are checked on the GPU in tests/test_gpu_mma_mutants.py."""

from __future__ import annotations

import numpy as np
import pytest

from mma_mutants import MMA_MUTANTS, grid, mma_mm, sizes


@pytest.mark.parametrize("mut,what,must_decline", MMA_MUTANTS, ids=[f"mut{m[0]}" for m in MMA_MUTANTS])
def test_proof_decisions(mut, what, must_decline):
    M, N, K = 40, 36, 48
    s = sizes(M, N, K)
    ck = mma_mm.compile(np.zeros(s["a"], np.float32), np.zeros(s["b"], np.float32), np.zeros(s["c"], np.float32),
                        M, N, K=K, MUT=mut)
    plan = ck.plan.native
    d = None if plan is None else plan.analyse({"M": M, "N": N}, grid(M, N), 0xFFFFFFFF)
    if mut == 0:
        assert d is not None and (d["M"], d["N"], d["K"]) == (M, N, K), plan.last_reason
    if must_decline:
        assert d is None, f"{what}: accepted"
