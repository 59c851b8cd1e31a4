"""GPU: the bounded waits of the native kernels expire into a status the host reads, without a
fault, trap or hang, and the context stays usable afterwards.

``eas_wait_selftest`` waits, with the GEMM's own bounded mbarrier wait, on a barrier that
nothing completes (budget ~5 ms); the status word then reads EAS_ERR_TIMEOUT."""

import ctypes
import time

import numpy as np
import pytest

from easy_as_b200.runtime import cuda_ext

pytestmark = pytest.mark.gpu


def _status(lib) -> int:
    code = ctypes.c_int()
    cuda_ext.check(lib.eas_gemm_status(0, ctypes.byref(code)), "status")
    return code.value


def test_expired_wait_sets_the_status_and_the_context_survives(cuda_rt):
    lib = cuda_ext.load()
    cuda_ext.check(lib.eas_set_device(0), "set_device")
    _status(lib)                                              # start from a clear word
    t0 = time.perf_counter()
    cuda_ext.check(lib.eas_wait_selftest(10_000_000, None), "wait selftest")
    cuda_ext.check(lib.eas_stream_synchronize(None), "sync")
    assert time.perf_counter() - t0 < 5.0
    assert _status(lib) == cuda_ext.EAS_ERR_TIMEOUT
    assert _status(lib) == 0                                  # reading clears it
    # the context is intact: a native GEMM right after is correct
    from examples.matmul_dot_f16 import grid, matmul_dot_f16

    rng = np.random.default_rng(0)
    M, N, K = 256, 256, 128
    a = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float16)
    c = np.zeros((M, N), np.float32)
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, _grid=grid(1))
    assert cuda_rt.native_launches == before + 1
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.abs(c - ref).max() <= 1e-5 * np.abs(ref).max()


def test_runtime_turns_an_expired_wait_into_an_error(cuda_rt):
    lib = cuda_ext.load()
    cuda_ext.check(lib.eas_set_device(0), "set_device")
    _status(lib)
    cuda_ext.check(lib.eas_wait_selftest(10_000_000, None), "wait selftest")
    cuda_ext.check(lib.eas_stream_synchronize(None), "sync")
    cuda_rt.native_launches += 1                              # as after a native launch
    with pytest.raises(RuntimeError, match="bounded pipeline wait expired"):
        cuda_rt._check_native_status(0)
    assert _status(lib) == 0
