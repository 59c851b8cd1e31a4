"""CPU: the elementwise analysis (which buffers a kernel loads, which it stores, and each store's
mask bound) on the variants of tests/ew_mutants.py.  The pipelined host path relies on it to skip
copies; tests/test_gpu_pipeline_mutants.py checks the host results on the GPU."""

from __future__ import annotations

import numpy as np
import pytest

from ew_mutants import EW_MUTANTS, ew_mut

EXPECTED = {
    0: (["a", "b"], [("c", ("arg", "N")), ("d", ("const", 1))]),
    3: (["a", "b"], [("c", ("arg", "M")), ("d", ("const", 1))]),
    4: (["a", "c"], [("c", ("arg", "N")), ("d", ("const", 1))]),   # b's load is dead code
    6: (["a", "b"], [("c", ("const", 1000)), ("d", ("const", 1))]),
    7: (["a", "b"], [("c", ("arg", "N")), ("d", ("arg", "M"))]),
}


@pytest.mark.parametrize("mut,what,elementwise", EW_MUTANTS, ids=[f"mut{m[0]}" for m in EW_MUTANTS])
def test_elementwise_analysis(mut, what, elementwise):
    x = np.zeros(100, np.float32)
    info = ew_mut.compile(x, x, x, x, 100, 50, MUT=mut, BLOCK=256).plan.elementwise
    assert (info is not None) == elementwise, what
    if info is not None:
        reads, bounds = EXPECTED[mut]
        assert sorted(info.reads) == reads
        assert sorted(info.store_bounds) == sorted(bounds)
