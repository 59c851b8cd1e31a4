"""GPU parity of the fp16 mk.dot GEMM pattern on the tcgen05 native kernel.

Tolerance: rtol 2e-2 against a float64 reference for fp16
GEMM with fp32 accumulation.  The tests also hold the native result to a much
tighter normwise bound against the CPU oracle's strictly ordered f32 fma chain
(the reference's dot semantics): max|gpu - oracle| <= 1e-5 * max|oracle|.
"""

import numpy as np
import pytest

from examples.matmul_dot_f16 import grid, matmul_dot_f16
from oracle.interp import execute

import eas
from eas import mk

pytestmark = pytest.mark.gpu


def _inputs(batch, M, N, K, seed=0):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((batch, M, K)) / np.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal((batch, K, N)) / np.sqrt(K)).astype(np.float16)
    return a, b


def _run(cuda_rt, batch, M, N, K, bn, seed=0):
    a, b = _inputs(batch, M, N, K, seed)
    c = np.zeros((batch, M, N), np.float32)
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=bn,
                   _grid=grid(batch))
    return a, b, c, cuda_rt.native_launches - before


def _ref64(a, b):
    return np.matmul(a.astype(np.float64), b.astype(np.float64))


@pytest.mark.parametrize("batch,M,N,K,bn", [(1, 256, 256, 64, 256), (1, 512, 512, 1024, 256),
                                            (1, 384, 640, 320, 128), (3, 200, 304, 136, 256),
                                            (2, 129, 264, 72, 128)])
def test_native_gemm_matches_fp64(cuda_rt, batch, M, N, K, bn):
    a, b, c, native = _run(cuda_rt, batch, M, N, K, bn)
    assert native == 1, "expected the tcgen05 path"
    ref = _ref64(a, b)
    np.testing.assert_allclose(c, ref, rtol=2e-2, atol=2e-2 * np.abs(ref).max())
    assert np.abs(c - ref).max() <= 1e-5 * np.abs(ref).max() + 1e-7


def test_native_gemm_matches_oracle(cuda_rt):
    batch, M, N, K = 2, 130, 264, 200
    a, b, c, native = _run(cuda_rt, batch, M, N, K, 256, seed=5)
    assert native == 1
    ck = matmul_dot_f16.compile(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_M=128, BLOCK_N=256,
                                BLOCK_K=64)
    want = np.zeros(batch * M * N, np.float32)
    execute(ck.ir, {"a": a.reshape(-1), "b": b.reshape(-1), "c": want, "M": M, "N": N, "K": K},
            grid=(-(-N // 256), M, batch))
    want = want.reshape(batch, M, N)
    assert np.abs(c - want).max() <= 1e-5 * np.abs(want).max()


def test_generic_path_equals_oracle_bitwise(cuda_rt, monkeypatch):
    """With the native kernel disabled the generic FFMA code reproduces the oracle bit for bit."""
    monkeypatch.setenv("EAS_DISABLE_NATIVE", "1")
    batch, M, N, K = 1, 33, 70, 45
    a, b, c, native = _run(cuda_rt, batch, M, N, K, 128, seed=2)
    assert native == 0
    ck = matmul_dot_f16.compile(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_M=128, BLOCK_N=128,
                                BLOCK_K=64)
    want = np.zeros(M * N, np.float32)
    execute(ck.ir, {"a": a.reshape(-1), "b": b.reshape(-1), "c": want, "M": M, "N": N, "K": K},
            grid=(1, M, batch))
    np.testing.assert_array_equal(c.reshape(-1), want)


def test_unaligned_n_is_repitched_and_runs_natively(cuda_rt):
    """N = 300: B rows are 600 bytes apart, not a TMA stride; B is re-pitched into scratch rows of 304
    elements (``eas_pad_f16_2d``) and the tcgen05 GEMM runs on the copy."""
    a, b, c, native = _run(cuda_rt, 3, 20, 300, 136, 256, seed=4)
    assert native == 1
    ref = _ref64(a, b)
    assert np.abs(c - ref).max() <= 1e-5 * np.abs(ref).max()


def test_unaligned_k_is_repitched_and_runs_natively(cuda_rt):
    """K = 45: A rows are 90 bytes apart; A (and B's 45 rows) are re-pitched; the padding is never
    read by the GEMM, which still runs K = 45."""
    a, b, c, native = _run(cuda_rt, 1, 40, 96, 45, 128, seed=3)
    assert native == 1
    ref = _ref64(a, b)
    assert np.abs(c - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("batch,M,N,K", [(4, 300, 1000, 1044), (2, 129, 203, 77)])
def test_unaligned_batched_shapes_match_float64(cuda_rt, batch, M, N, K):
    """Batched launches whose pitches TMA cannot use (K = 1044: 2088-byte A rows; odd N) run natively
    on re-pitched operands."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(K)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=256, _grid=grid(batch))
    assert cuda_rt.native_launches == before + 1
    ref = torch.bmm(a.double(), b.double())
    assert ((c.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-5


@eas.kernel
def gemm_nt(a, b, c, M, N, K, BLOCK: eas.constexpr):
    col = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    row = mk.program_id(1)
    inside = (row < M) & (col < N)
    mk.store(c, row * N + col, mk.dot(a, row * K, 1, b, col * K, 1, mk.where(inside, K, 0)), inside)


@pytest.mark.parametrize("bn", [128, 256])
def test_native_gemm_k_major_b(cuda_rt, bn):
    M, N, K = 300, 520, 192
    rng = np.random.default_rng(9)
    a = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    bt = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)  # B stored as [N, K]
    c = np.zeros((M, N), np.float32)
    before = cuda_rt.native_launches
    gemm_nt(a.reshape(-1), bt.reshape(-1), c.reshape(-1), M, N, K, BLOCK=bn, _grid=(-(-N // bn), M, 1))
    assert cuda_rt.native_launches - before == 1
    ref = a.astype(np.float64) @ bt.astype(np.float64).T
    assert np.abs(c - ref).max() <= 1e-5 * np.abs(ref).max()


def test_torch_tensors_zero_copy_and_async(cuda_rt):
    import torch

    batch, M, N, K = 4, 256, 512, 2088  # the C5 runtime-K tail (2088 = 32*64 + 40)
    g = torch.Generator(device="cuda").manual_seed(4)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.empty(batch, M, N, device="cuda")
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=256,
                   _grid=grid(batch), _sync=False)
    cuda_rt.synchronize()
    ref = torch.bmm(a.double(), b.double())
    assert ((c.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-5
