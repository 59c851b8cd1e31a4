"""The allocation-free GEMM entry point gives the same results as the regular one.

eas_gemm_f16_noalloc exists for callers that cannot let a library allocate
memory (their own allocator owns every byte, or allocating at launch time is
not allowed): its status word sits in a fixed device array of the library
instead of memory allocated on first use.  This file is collected last so that
a failure here never hides the other tests.
"""

import ctypes

import pytest

from easy_as_b200.runtime import cuda_ext

pytestmark = pytest.mark.gpu


def _gemm(lib, fn, a, b, c, batch, M, N, K, status=None):
    args = [a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, batch, K, M * K, N, K * N, 0, N, M * N, 256, 0]
    if status is not None:
        args.append(ctypes.byref(status))
    rc = fn(*args)
    assert rc == 0, cuda_ext.last_error()


@pytest.mark.parametrize("shape", [(2, 200, 264, 136), (1, 256, 512, 2088)])
def test_noalloc_matches_regular_entry_point_twice(cuda_rt, shape):
    import torch

    lib = cuda_ext.load()
    batch, M, N, K = shape
    for call in range(2):  # the shared status word must be cleared between calls
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
        b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
        want = torch.zeros(batch, M, N, device="cuda")
        got = torch.full((batch, M, N), float("nan"), device="cuda")
        _gemm(lib, lib.eas_gemm_f16, a, b, want, batch, M, N, K)
        status = ctypes.c_int(-1)
        _gemm(lib, lib.eas_gemm_f16_noalloc, a, b, got, batch, M, N, K, status)
        torch.cuda.synchronize()
        assert status.value == 0
        scale = want.abs().max().item()
        assert (got - want).abs().max().item() <= 1e-5 * scale
        ref = torch.bmm(a.double(), b.double())
        assert ((got.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-5


def test_noalloc_rejects_oversized_dimensions(cuda_rt):
    lib = cuda_ext.load()
    dummy = ctypes.c_void_p(256)
    rc = lib.eas_gemm_f16_noalloc(dummy, dummy, dummy, 1 << 31, 8, 8, 1, 8, 0, 8, 0, 0, 8, 0, 256, None, None)
    assert rc == cuda_ext.EAS_ERR_VALUE
    assert "2^31" in cuda_ext.last_error()


@pytest.mark.parametrize("block_n", [128, 256])
@pytest.mark.parametrize("b_kmajor", [0, 1])
@pytest.mark.parametrize("ldc_pad", [0, 1])
def test_noalloc_layouts_match_regular_entry_point(cuda_rt, block_n, b_kmajor, ldc_pad):
    """Both N tiles, N-major and K-major B, and a C whose rows are not 16-byte strided (ldc = N + 1:
    the kernel's direct-store epilogue instead of TMA stores), each called twice in a row."""
    import torch

    lib = cuda_ext.load()
    batch, M, N, K = 2, 136, 264, 200
    ldc = N + ldc_pad
    for call in range(2):
        g = torch.Generator(device="cuda").manual_seed(7 + call)
        a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
        b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
        bop = b.transpose(1, 2).contiguous() if b_kmajor else b
        ldb = K if b_kmajor else N
        outs = []
        for fn in (lib.eas_gemm_f16, lib.eas_gemm_f16_noalloc):
            c = torch.full((batch, M, ldc), float("nan"), device="cuda")
            args = [a.data_ptr(), bop.data_ptr(), c.data_ptr(), M, N, K, batch, K, M * K, ldb, K * N, b_kmajor, ldc,
                    M * ldc, block_n, 0]
            status = ctypes.c_int(-1)
            if fn is lib.eas_gemm_f16_noalloc:
                args.append(ctypes.byref(status))
            assert fn(*args) == 0, cuda_ext.last_error()
            torch.cuda.synchronize()
            if fn is lib.eas_gemm_f16_noalloc:
                assert status.value == 0
            outs.append(c[:, :, :N])
        want, got = outs
        assert not torch.isnan(got).any()
        assert (got - want).abs().max().item() <= 1e-5 * want.abs().max().item()
