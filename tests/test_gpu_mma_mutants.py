"""GPU: every near-miss variant of the DSL simdgroup-MMA matmul (tests/mma_mutants.py) computes what
the mutant says, native (f16 staging + tcgen05) or generated (mma.sync): within 1e-5 normwise of
the oracle, which sums each 8x8 mma step in float64 and rounds once (the summation order of the
matrix units is unspecified, so neither GPU path is bound to the oracle's)."""

from __future__ import annotations

import numpy as np
import pytest

from mma_mutants import MMA_MUTANTS, grid, mma_mm, sizes
from oracle.interp import execute

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mut,what,must_decline", MMA_MUTANTS, ids=[f"mut{m[0]}" for m in MMA_MUTANTS])
@pytest.mark.parametrize("M,N,K", [(40, 36, 48), (100, 70, 64)])
def test_mma_mutant_vs_oracle(cuda_rt, mut, what, must_decline, M, N, K):
    s = sizes(M, N, K)
    rng = np.random.default_rng(mut * 10 + M)
    a = rng.standard_normal(s["a"]).astype(np.float32)
    b = rng.standard_normal(s["b"]).astype(np.float32)
    c0 = rng.standard_normal(s["c"]).astype(np.float32)
    gpu, cpu = c0.copy(), c0.copy()
    before = cuda_rt.native_launches
    mma_mm(a, b, gpu, M, N, K=K, MUT=mut, _grid=grid(M, N))
    native = cuda_rt.native_launches - before
    assert not (must_decline and native), f"{what}: ran natively"
    if mut == 0:
        assert native, "the unchanged kernel should run on the native path"
    ck = mma_mm.compile(a, b, cpu, M, N, K=K, MUT=mut)
    execute(ck.ir, {"a": a, "b": b, "c": cpu, "M": M, "N": N}, grid=grid(M, N))
    err = np.abs(gpu.astype(np.float64) - cpu).max() / np.abs(cpu).max()
    assert err <= 1e-5, f"{what} ({'native' if native else 'generated'}): normwise error {err:.2e}"
