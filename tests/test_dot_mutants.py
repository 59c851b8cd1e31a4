"""CPU: the fp16 dot-GEMM pattern (and, where it does not match, the tiled-GEMM proof) on near-miss
variants of the dot GEMM kernel (tests/dot_mutants.py): the unchanged kernel is accepted, every
mutant that is not a GEMM in a layout the native kernels take is declined.  What accepted
mutants compute is checked on the GPU in tests/test_gpu_dot_mutants.py."""

from __future__ import annotations

import numpy as np
import pytest

from dot_mutants import DOT_MUTANTS, dot_mut, grid, sizes

ALL_THREADS = 0xFFFFFFFF


def decision(mut, batch, M, N, K):
    """(accepted, reason) of the native plan for one launch."""
    s = sizes(mut, batch, M, N, K)
    ck = dot_mut.compile(np.zeros(s["a"], np.float16), np.zeros(s["b"], np.float16), np.zeros(s["c"], np.float32),
                         M, N, K, MUT=mut)
    plan = ck.plan.native
    if plan is None:
        return False, "no native plan"
    if hasattr(plan, "map_launch"):
        scal = {f"${a.name}": v for a, v in zip([a for a in ck.ir.args if a.kind == "scalar"], (M, N, K))}
        m = plan.map_launch(scal, grid(batch, M, N), ALL_THREADS)
    else:
        m = plan.analyse({"M": M, "N": N, "K": K}, grid(batch, M, N), ALL_THREADS)
    return m is not None, plan.last_reason


@pytest.mark.parametrize("mut,what,must_decline", DOT_MUTANTS, ids=[f"mut{m[0]}" for m in DOT_MUTANTS])
def test_pattern_decisions(mut, what, must_decline):
    ok, reason = decision(mut, 2, 200, 264, 136)
    if mut == 0:
        assert ok, reason
    if must_decline:
        assert not ok, f"{what}: accepted"
