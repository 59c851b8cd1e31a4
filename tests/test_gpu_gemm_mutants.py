"""GPU: every near-miss variant of the tiled matmul (tests/gemm_mutants.py) gives the oracle's bits,
whether the tiled-GEMM proof accepted it (native FFMA kernel) or declined it (generated kernel)."""

from __future__ import annotations

import numpy as np
import pytest

from gemm_mutants import MUTANTS, grid, sizes, tile_mm_mut
from oracle.interp import execute

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mut,what,must_decline", MUTANTS, ids=[f"mut{m[0]}" for m in MUTANTS])
@pytest.mark.parametrize("M,N,K", [(70, 90, 48), (64, 64, 40), (33, 130, 64)])
def test_mutant_bit_exact_vs_oracle(cuda_rt, mut, what, must_decline, M, N, K):
    s = sizes(mut, M, N, K)
    rng = np.random.default_rng(mut * 1000 + M)
    a = rng.standard_normal(s["a"]).astype(np.float32)
    b = rng.standard_normal(s["b"]).astype(np.float32)
    c0 = rng.standard_normal(s["c"]).astype(np.float32)      # mutant 10 reads C; others keep unwritten C
    gpu, cpu = c0.copy(), c0.copy()
    before = cuda_rt.native_launches
    tile_mm_mut(a, b, gpu, M, N, K=K, MUT=mut, _grid=grid(M, N))
    native = cuda_rt.native_launches - before
    assert not (must_decline and native), f"{what}: ran natively"
    ck = tile_mm_mut.compile(a, b, cpu, M, N, K=K, MUT=mut)
    execute(ck.ir, {"a": a, "b": b, "c": cpu, "M": M, "N": N}, grid=grid(M, N))
    bad = np.nonzero(gpu.view(np.uint32) != cpu.view(np.uint32))[0]
    assert bad.size == 0, (f"{what} ({'native' if native else 'generated'}): {bad.size} differ, first at "
                           f"{bad[0]}: gpu {gpu[bad[0]]!r} oracle {cpu[bad[0]]!r}")
