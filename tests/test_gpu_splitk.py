"""GPU: split-K in the tcgen05 GEMMs (CTA-pair kernel, and the 1-SM kernel that M <= 128 uses).

Launches with at most half as many 256x256 tiles as CTA pairs split each tile's K range into
2 parts (4 with EAS_GEMM_SPLITK=4), summed into a zeroed C with TMA reduce-adds.  The small and ragged launches here
split; the per-GPU shards of config C4 at 4 and 8 GPUs (256 and 128 tiles) do not, and stay as
regression cases for the multi-wave schedule.  Each result is held to the fp16 GEMM bound
against float64 (rtol 2e-2) through a normwise bound of max(1e-5, 4e-9 K)."""

from __future__ import annotations

import pytest

from examples.matmul_dot_f16 import grid, matmul_dot_f16

pytestmark = pytest.mark.gpu


def _gemm(cuda_rt, batch, M, N, K, seed, bn=256):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=bn,
                   _grid=grid(batch), _sync=True)
    assert cuda_rt.native_launches == before + 1
    return a, b, c


@pytest.mark.parametrize("batch,M,N,K,bn", [(1, 1024, 8192, 8192, 256), (1, 2048, 8192, 8192, 256),
                                            (1, 512, 512, 4096, 256), (2, 512, 768, 2048, 256),
                                            (1, 700, 1000, 3000, 256),
                                            # M <= 128: the 1-SM kernel, split over the SMs
                                            (1, 128, 8192, 8192, 256), (1, 64, 4096, 2048, 128),
                                            (3, 100, 1000, 1024, 128)])
def test_split_k_matches_float64(cuda_rt, batch, M, N, K, bn):
    import torch

    a, b, c = _gemm(cuda_rt, batch, M, N, K, seed=M + K, bn=bn)
    ref = torch.bmm(a.double(), b.double())
    err = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    # f32 accumulation in the tensor core: the normwise error grows with K (1.07e-5 at K = 8192 unsplit)
    assert err <= max(1e-5, 4e-9 * K), err
    assert not torch.isnan(c).any()


@pytest.mark.parametrize("batch,M,N,K,bn", [(1, 512, 512, 4096, 256), (1, 128, 8192, 8192, 256),
                                            (1, 64, 4096, 2048, 128)])
def test_default_split_k_is_bit_reproducible(cuda_rt, batch, M, N, K, bn):
    """The default split (2 parts, M = 128 and smaller launches included) gives the same bits on
    every run: (0 + p) + q and (0 + q) + p are both exactly p + q."""
    import ctypes

    import torch

    from easy_as_b200.runtime import cuda_ext

    _, _, first = _gemm(cuda_rt, batch, M, N, K, seed=9, bn=bn)
    vals = [ctypes.c_int() for _ in range(6)]
    cuda_ext.load().eas_gemm_last_config(*(ctypes.byref(v) for v in vals))
    assert vals[3].value == 2, "expected a 2-way split launch"
    for _ in range(9):
        _, _, again = _gemm(cuda_rt, batch, M, N, K, seed=9, bn=bn)
        assert torch.equal(first.view(torch.int32), again.view(torch.int32))


@pytest.mark.parametrize("batch,M,N,K,bn", [(1, 8192, 8192, 1024, 256), (1, 512, 512, 4096, 256),
                                            (1, 128, 8192, 8192, 256), (2, 300, 1000, 520, 128)])
def test_launch_matches_the_plan_query(cuda_rt, batch, M, N, K, bn):
    """eas_gemm_f16_plan predicts what eas_gemm_f16 launches (checked against the tile configuration
    the launch recorded)."""
    import ctypes

    import torch

    from easy_as_b200.runtime import cuda_ext

    _gemm(cuda_rt, batch, M, N, K, seed=1, bn=bn)
    lib = cuda_ext.load()
    got = [ctypes.c_int() for _ in range(6)]
    lib.eas_gemm_last_config(*(ctypes.byref(v) for v in got))
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    want = [ctypes.c_int() for _ in range(6)]
    cuda_ext.check(lib.eas_gemm_f16_plan(M, N, K, batch, bn, 0, 0, 1, sms, sms // 2,
                                         *(ctypes.byref(v) for v in want)), "plan")
    assert [v.value for v in got] == [v.value for v in want]
