"""GPU: every explicit tile configuration of the fp16 dot GEMM (``eas_gemm_f16_tile``), i.e. the
autotune space BLOCK_M x BLOCK_N x BLOCK_K = {128, 256} x {128, 256} x {64, 128} of config C4,
launches the kernel it names and matches float64 within the fp16 GEMM bound (normwise
``max(1e-5, 4e-9 K)``, the split-K tests' bound; rtol 2e-2 is the north-star tolerance).

Ragged M, N and K are included: with BLOCK_K = 128 an odd number of 64-deep k-blocks leaves the
last stage half past K, which TMA fills with zeros."""

from __future__ import annotations

import ctypes

import pytest

from examples.matmul_dot_f16 import CONFIGS, grid, matmul_dot_f16, matmul_dot_f16_tuned

pytestmark = pytest.mark.gpu

SPACE = [(bm, bn, bk) for bm in (128, 256) for bn in (128, 256) for bk in (64, 128)]


def _last():
    from easy_as_b200.runtime import cuda_ext

    vals = [ctypes.c_int() for _ in range(6)]
    cuda_ext.check(cuda_ext.load().eas_gemm_last_config(*(ctypes.byref(v) for v in vals)), "last config")
    tm, tn, st, ks, pair, bk = (v.value for v in vals)
    return {"tile": (tm, tn), "stages": st, "ksplit": ks, "pair": bool(pair), "block_k": bk}


def _operands(batch, M, N, K, seed):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    return a, b


@pytest.mark.parametrize("bm,bn,bk", SPACE)
@pytest.mark.parametrize("batch,M,N,K", [(1, 1024, 1536, 1024), (2, 300, 704, 200), (1, 513, 1000, 2088)])
def test_each_tile_config_matches_float64(cuda_rt, bm, bn, bk, batch, M, N, K):
    import torch

    a, b = _operands(batch, M, N, K, seed=M + N + K)
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk,
                   _grid=grid(batch), _sync=True)
    assert cuda_rt.native_launches == before + 1
    cfg = _last()
    assert cfg["pair"] == (bm == 256)
    assert cfg["block_k"] == bk
    assert cfg["tile"] == ((128, bn) if bm == 128 else (256, 2 * bn))
    ref = torch.bmm(a.double(), b.double())
    err = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    assert not torch.isnan(c).any()
    assert err <= max(1e-5, 4e-9 * K), err


@pytest.mark.parametrize("bm,bn,bk", [(128, 128, 128), (256, 128, 128), (256, 256, 128)])
def test_k_major_b_with_two_k_blocks_per_stage(cuda_rt, bm, bn, bk):
    """B stored [N, K] (K-major descriptors) through the C entry point."""
    import torch

    from easy_as_b200.runtime import cuda_ext

    batch, M, N, K = 2, 520, 1032, 712      # 712 = 11 k-blocks + 8: odd count, ragged tail
    a, b = _operands(batch, M, N, K, seed=7)
    bt = b.transpose(1, 2).contiguous()
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    rc = cuda_ext.load().eas_gemm_f16_tile(a.data_ptr(), bt.data_ptr(), c.data_ptr(), M, N, K, batch, K, M * K, K,
                                           N * K, 1, N, M * N, bm, bn, bk, None)
    cuda_ext.check(rc, "eas_gemm_f16_tile")
    torch.cuda.synchronize()
    assert _last()["block_k"] == bk
    ref = torch.bmm(a.double(), b.double())
    assert ((c.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-5


def test_autotune_picks_the_fastest_of_eight_kernels_at_c4(cuda_rt):
    """C4 (8192^3): the tuner times the eight configs (eight different kernels) and keeps the one
    with the smallest measured time."""
    import torch

    M = N = K = 8192
    a, b = _operands(1, M, N, K, seed=3)
    c = torch.empty(M * N, device="cuda")
    k = matmul_dot_f16_tuned
    k._tuned_cache.clear()
    k._tuned_times.clear()
    import os

    old = os.environ.get("EAS_AUTOTUNE_CACHE")
    os.environ["EAS_AUTOTUNE_CACHE"] = "0"
    try:
        k(a.reshape(-1), b.reshape(-1), c, M, N, K, _grid=grid(1), _sync=True)
    finally:
        if old is None:
            os.environ.pop("EAS_AUTOTUNE_CACHE", None)
        else:
            os.environ["EAS_AUTOTUNE_CACHE"] = old
    (times,) = k._tuned_times.values()
    assert [t[0] for t in times] == [dict(cfg.meta) for cfg in CONFIGS]
    assert all(t[1] > 0 for t in times)
    (best,) = k._tuned_cache.values()
    assert dict(best.meta) == min(times, key=lambda t: t[1])[0]
    ref = a[0, :2].double() @ b[0].double()
    assert ((c.view(M, N)[:2].double() - ref).abs().max() / ref.abs().max()).item() <= 1e-4
