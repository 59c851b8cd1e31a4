"""GPU: every near-miss variant of the fp16 dot GEMM (tests/dot_mutants.py) computes what the
mutant says.  A launch the native tcgen05 kernel took is held to 1e-5 normwise of the oracle's
ordered f32 fma chains (the tensor core sums in another order); a launch that ran the generated
kernel matches the oracle bit for bit.  Unwritten parts of C keep their prior contents."""

from __future__ import annotations

import numpy as np
import pytest

from dot_mutants import DOT_MUTANTS, dot_mut, grid, sizes
from oracle.interp import execute

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mut,what,must_decline", DOT_MUTANTS, ids=[f"mut{m[0]}" for m in DOT_MUTANTS])
@pytest.mark.parametrize("batch,M,N,K", [(2, 200, 264, 136), (1, 130, 520, 72)])
def test_dot_mutant_vs_oracle(cuda_rt, mut, what, must_decline, batch, M, N, K):
    s = sizes(mut, batch, M, N, K)
    rng = np.random.default_rng(mut * 100 + M)
    a = (rng.standard_normal(s["a"]) / np.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal(s["b"]) / np.sqrt(K)).astype(np.float16)
    c0 = rng.standard_normal(s["c"]).astype(np.float32)
    gpu, cpu = c0.copy(), c0.copy()
    before = cuda_rt.native_launches
    dot_mut(a, b, gpu, M, N, K, MUT=mut, _grid=grid(batch, M, N))
    native = cuda_rt.native_launches - before
    assert not (must_decline and native), f"{what}: ran natively"
    ck = dot_mut.compile(a, b, cpu, M, N, K, MUT=mut)
    execute(ck.ir, {"a": a, "b": b, "c": cpu, "M": M, "N": N, "K": K}, grid=grid(batch, M, N))
    if native:
        err = np.abs(gpu.astype(np.float64) - cpu).max() / np.abs(cpu).max()
        assert err <= 1e-5, f"{what} (native): normwise error {err:.2e}"
    else:
        bad = np.nonzero(gpu.view(np.uint32) != cpu.view(np.uint32))[0]
        assert bad.size == 0, f"{what} (generated): {bad.size} differ, first at {bad[0]}"
