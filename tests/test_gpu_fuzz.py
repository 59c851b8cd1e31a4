"""GPU: random DSL kernels (tests/fuzz_kernels.py) run through the CUDA lowering give the same bits
as the CPU oracle on the same inputs: f32 and f16 arithmetic, u32 index math, casts, masks and
zero-filled masked loads at shifted and permuted offsets.  Sizes include ragged tails.

One allowance: IEEE 754 leaves the sign and payload of a NaN produced by an invalid operation
(inf * 0, inf - inf) unspecified, and the GPU returns the canonical 0x7fffffff where x86 numpy
returns 0xffc00000; a NaN matches any NaN (as ``assert_allclose`` treats them in the
reference's tests).  Every other value, -0.0 and infinities included, must match bit for bit."""

from __future__ import annotations

import numpy as np
import pytest

import fuzz_kernels
from oracle.interp import execute

pytestmark = pytest.mark.gpu

SEEDS = range(80)


@pytest.mark.parametrize("seed", SEEDS)
def test_fuzz_kernel_bit_exact_vs_oracle(cuda_rt, seed):
    k, src = fuzz_kernels.make(seed)
    n = 1000 + 37 * seed
    block = (64, 128, 256, 1024)[seed % 4]
    gpu = fuzz_kernels.inputs(seed, n)
    cpu = fuzz_kernels.inputs(seed, n)
    names = ("x", "y", "h", "out", "outi", "outh", "N", "S", "alpha")
    k(*(gpu[a] for a in names), BLOCK=block)
    ck = k.compile(*(cpu[a] for a in names), BLOCK=block)
    execute(ck.ir, dict(cpu), grid=(-(-n // block), 1, 1))
    for buf in ("out", "outi", "outh"):
        bits = np.uint16 if gpu[buf].dtype == np.float16 else np.uint32
        g, c = gpu[buf].view(bits), cpu[buf].view(bits)
        both_nan = np.isnan(gpu[buf]) & np.isnan(cpu[buf])
        bad = np.nonzero((g != c) & ~both_nan)[0]
        assert bad.size == 0, (f"{buf}: {bad.size} of {n} differ, first at {bad[0]}: gpu {gpu[buf][bad[0]]!r} "
                               f"oracle {cpu[buf][bad[0]]!r}\n{src}")


@pytest.mark.parametrize("seed", range(60))
def test_thread_fuzz_kernel_bit_exact_vs_oracle(cuda_rt, seed):
    """Thread-mode kernels (threadgroup memory, barriers, fma chains, mk.dot): bit-exact against the
    oracle.  None of them is a GEMM, so the tiled-GEMM proof, which examines every thread-mode
    kernel with fma or dot, must decline them all; a wrongly accepted kernel would show as a
    mismatch here."""
    k, src, meta = fuzz_kernels.make_thread(seed)
    n = 700 + 29 * seed
    gpu = fuzz_kernels.thread_inputs(seed, n)
    cpu = fuzz_kernels.thread_inputs(seed, n)
    names = ("x", "y", "out", "N", "S", "alpha")
    grid = (-(-n // meta["NT"]), 1, 1)
    before = cuda_rt.native_launches
    k(*(gpu[a] for a in names), _grid=grid, **meta)
    assert cuda_rt.native_launches == before, "a random thread kernel was launched as a native GEMM"
    ck = k.compile(*(cpu[a] for a in names), **meta)
    execute(ck.ir, dict(cpu), grid=grid)
    g, c = gpu["out"].view(np.uint32), cpu["out"].view(np.uint32)
    both_nan = np.isnan(gpu["out"]) & np.isnan(cpu["out"])
    bad = np.nonzero((g != c) & ~both_nan)[0]
    assert bad.size == 0, (f"{bad.size} of {n} differ, first at {bad[0]}: gpu {gpu['out'][bad[0]]!r} "
                           f"oracle {cpu['out'][bad[0]]!r}\n{src}")
