"""CPU: mk.mma on f32 operands (the reference's simdgroup_float8x8 path, eas/codegen/msl.py:970-980).

No reference test pins it, so the oracle's f32 fragment semantics (8x8 tiles loaded with a row
stride, D = A @ B + C in f32) are pinned here against float64 numpy, for a K loop of several
steps and for a C tile that starts from a loaded accumulator; and its lowering compiles in both
the plain and the bounds-checked mode."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import eas
from eas import mk
from easy_as_b200.codegen.cuda import ir_to_cuda
from easy_as_b200.runtime import cuda_ext
from oracle.interp import execute


@eas.kernel
def mma_f32(a, b, c, K: eas.constexpr, N: eas.constexpr):
    """One simdgroup: C (8 x N, stride N) = A (8 x K, stride K) @ B (K x N, stride N), one 8x8
    column block of C per k loop."""
    _t = mk.tid(0, 32)
    for n0 in range(0, N, 8):
        acc = mk.mma_zero()
        for k0 in range(0, K, 8):
            acc = mk.mma(a, k0, K, b, k0 * N + n0, N, acc)
        mk.mma_store(c, n0, N, acc)


@pytest.mark.parametrize("K,N", [(8, 8), (32, 16), (64, 24)])
def test_oracle_f32_mma_is_a_matmul(K, N):
    rng = np.random.default_rng(K + N)
    a = rng.standard_normal(8 * K).astype(np.float32)
    b = rng.standard_normal(K * N).astype(np.float32)
    c = np.zeros(8 * N, np.float32)
    ck = mma_f32.compile(a, b, c, K=K, N=N)
    execute(ck.ir, {"a": a, "b": b, "c": c}, grid=(1, 1, 1))
    ref = a.reshape(8, K).astype(np.float64) @ b.reshape(K, N).astype(np.float64)
    np.testing.assert_allclose(c.reshape(8, N), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("checked", [False, True])
def test_f32_mma_lowering_compiles(checked):
    a = np.zeros(8 * 32, np.float32)
    b = np.zeros(32 * 16, np.float32)
    c = np.zeros(8 * 16, np.float32)
    lo = ir_to_cuda(mma_f32.compile(a, b, c, K=32, N=16).ir, checked=checked)
    assert "eas_mma_f16(" not in lo.src.split("extern \"C\"")[1]   # f32 operands: the FFMA form
    lib = cuda_ext.load()
    img, size = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.eas_compile(lo.src.encode(), (lo.kernel_name + ".cu").encode(), None, 0, ctypes.byref(img),
                         ctypes.byref(size))
    assert rc == 0, cuda_ext.last_error()
    lib.eas_free_host(img)
