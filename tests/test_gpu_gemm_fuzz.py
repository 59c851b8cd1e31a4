"""GPU: the fp16 GEMM path on random shapes through the public API.

Sixty seeded shapes (batch 1-3, M 1-1100, N and K multiples of 8 up to 1600 and 1100, BLOCK_N
128 or 256, B row-major through the DSL kernel or K-major through the C entry point) exercise
the launcher's choices together: 1-SM or CTA-pair kernel, 256 x 256 or 256 x 512 tiles,
split-K, TMA-stored or directly stored C.  Every result is held to max(1e-5, 4e-9 K)
normwise against float64 (the tensor core's f32 accumulation), and no NaN may survive from
the prefilled output."""

from __future__ import annotations

import ctypes
import random

import pytest

from easy_as_b200.runtime import cuda_ext
from examples.matmul_dot_f16 import grid, matmul_dot_f16

pytestmark = pytest.mark.gpu


def _shape(i):
    r = random.Random(1000 + i)
    batch = r.choice([1, 1, 2, 3])
    M = r.choice([1, 7, 64, 128, 129, 255, 256, 300, 513, 1100])
    N = 8 * r.randint(1, 200)
    K = 8 * r.randint(1, 137)
    return batch, M, N, K, r.choice([128, 256]), r.random() < 0.3


@pytest.mark.parametrize("i", range(60))
def test_random_gemm_shapes(cuda_rt, i):
    import torch

    batch, M, N, K, bn, kmajor = _shape(i)
    g = torch.Generator(device="cuda").manual_seed(i)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    if kmajor:
        bt = b.transpose(1, 2).contiguous()
        lib = cuda_ext.load()
        rc = lib.eas_gemm_f16(a.data_ptr(), bt.data_ptr(), c.data_ptr(), M, N, K, batch, K, M * K, K, N * K, 1, N,
                              M * N, bn, None)
        cuda_ext.check(rc, "gemm_f16")
        torch.cuda.synchronize()
        code = ctypes.c_int()
        cuda_ext.check(lib.eas_gemm_status(0, ctypes.byref(code)), "status")
        assert code.value == 0
    else:
        matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=bn,
                       _grid=grid(batch), _sync=True)
    ref = torch.bmm(a.double(), b.double())
    assert not torch.isnan(c).any(), (batch, M, N, K, bn, kmajor)
    err = ((c.double() - ref).abs().max() / ref.abs().max().clamp_min(1e-30)).item()
    assert err <= max(1e-5, 4e-9 * K), (batch, M, N, K, bn, kmajor, err)
