"""CPU: the tiled-GEMM proof on near-miss variants of a tiled matmul (tests/gemm_mutants.py).
The unchanged kernel is proven a GEMM; every mutant that is not a GEMM in a layout the native
kernel takes is declined.  (What the accepted mutants compute is checked on the GPU, bit for
bit against the oracle, in tests/test_gpu_gemm_mutants.py.)"""

from __future__ import annotations

import numpy as np
import pytest

from gemm_mutants import MUTANTS, grid, sizes, tile_mm_mut

ALL_THREADS = 0xFFFFFFFF


def _plan(mut, M, N, K):
    s = sizes(mut, M, N, K)
    ck = tile_mm_mut.compile(np.zeros(s["a"], np.float32), np.zeros(s["b"], np.float32),
                             np.zeros(s["c"], np.float32), M, N, K=K, MUT=mut)
    return ck.plan.native


@pytest.mark.parametrize("mut,what,must_decline", MUTANTS, ids=[f"mut{m[0]}" for m in MUTANTS])
@pytest.mark.parametrize("M,N,K", [(70, 90, 48), (64, 64, 40)])
def test_proof_decisions(mut, what, must_decline, M, N, K):
    plan = _plan(mut, M, N, K)
    d = None if plan is None else plan.analyse({"M": M, "N": N}, grid(M, N), ALL_THREADS)
    if mut == 0:
        assert d is not None, plan.last_reason
    if must_decline:
        assert d is None, f"{what}: accepted as {d}"
