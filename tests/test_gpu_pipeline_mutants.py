"""GPU: every elementwise-kernel variant (tests/ew_mutants.py) run on page-locked host tensors gives
the oracle's bits for every host element, including the ones the kernel never stores.  The
pipelined copy path (copy in only loaded buffers, copy back only elements below the store bounds,
here forced onto small arrays in many chunks) must either be declined or be exact."""

from __future__ import annotations

import numpy as np
import pytest

from ew_mutants import EW_MUTANTS, ew_mut
from oracle.interp import execute

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mut,what,elementwise", EW_MUTANTS, ids=[f"mut{m[0]}" for m in EW_MUTANTS])
def test_pipelined_host_path_vs_oracle(cuda_rt, monkeypatch, mut, what, elementwise):
    import torch

    from easy_as_b200.runtime.cuda import CudaRuntime

    monkeypatch.setenv("EAS_PIPELINE_MIN_BYTES", "0")
    monkeypatch.setattr(CudaRuntime, "PIPELINE_CHUNK_ELEMS", 1 << 12)   # many chunks
    n, m_bound, block = 50_000 + 17, 31_111, 256
    rng = np.random.default_rng(mut)
    host = {k: torch.from_numpy(rng.standard_normal(n).astype(np.float32)).pin_memory() for k in "abcd"}
    cpu = {k: v.numpy().copy() for k, v in host.items()}
    ck = ew_mut.compile(*(cpu[k] for k in "abcd"), n, m_bound, MUT=mut, BLOCK=block)
    assert (ck.plan.elementwise is not None) == elementwise, what
    ew_mut(*(host[k] for k in "abcd"), n, m_bound, MUT=mut, BLOCK=block)
    execute(ck.ir, {**cpu, "N": n, "M": m_bound}, grid=(-(-n // block), 1, 1))
    for k in "abcd":
        got, want = host[k].numpy().view(np.uint32), cpu[k].view(np.uint32)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, f"{what}: {k} differs at {bad.size} elements, first {bad[0]}"
