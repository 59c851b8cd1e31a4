"""GPU: program-id sub-ranges (one rank's share of a multi-GPU launch, ``shard.run_shard`` /
``CudaRuntime.run_range``) take the native GEMM kernels and reproduce the full launch."""

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from easy_as_b200.shard import run_shard
from examples.matmul_dot_f16 import grid, matmul_dot_f16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,axis", [(2, 1), (3, 1), (4, 2)])
def test_f16_dot_gemm_shards_run_natively(cuda_rt, world, axis):
    import torch

    batch, M, N, K = 4, 512, 384, 264
    g = torch.Generator(device="cuda").manual_seed(1)
    a = (torch.randn(batch * M * K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch * K * N, device="cuda", generator=g) / K ** 0.5).half()
    full = torch.zeros(batch * M * N, device="cuda")
    meta = dict(BLOCK_N=256)
    matmul_dot_f16(a, b, full, M, N, K, **meta, _grid=grid(batch))
    parts = torch.zeros_like(full)
    before = cuda_rt.native_launches
    for r in range(world):
        run_shard(matmul_dot_f16, a, b, parts, M, N, K, **meta, _grid=grid(batch), _rank=r, _world=world,
                  _axis=axis)
    assert cuda_rt.native_launches == before + world
    # rows along the y axis, batches along z: every output tile is computed the same way
    torch.testing.assert_close(parts, full, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("slices", [False, True])
def test_tiled_fp32_shards_run_natively_bit_for_bit(cuda_rt, slices):
    import torch

    c = goldens.case("matmul_tiled_c3_full")
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    M = N = 512
    K = 2048
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.randn(M * K, device="cuda", generator=g)
    b = torch.randn(K * N, device="cuda", generator=g)
    full = torch.zeros(M * N, device="cuda")
    grid_ = (N // 32, M // 32, 1)
    cuda_rt.run(ck, {"a": a, "b": b, "c": full, "M": M, "N": N}, c["meta"], grid=grid_)
    out = torch.zeros(M * N, device="cuda")
    before = cuda_rt.native_launches
    for lo, hi in ((0, 5), (5, 16)):                # program rows 0..4 and 5..15 (32 rows each)
        if slices:
            # each part holds only its rows of A and C
            a_part = a[lo * 32 * K: hi * 32 * K].clone()
            c_part = torch.zeros((hi - lo) * 32 * N, device="cuda")
            cuda_rt.run_range(ck, {"a": a_part, "b": b, "c": c_part, "M": M, "N": N}, c["meta"], axis=1, lo=lo, hi=hi,
                              grid=grid_, buffer_base={"a": lo * 32 * K, "c": lo * 32 * N})
            out[lo * 32 * N: hi * 32 * N] = c_part
        else:
            cuda_rt.run_range(ck, {"a": a, "b": b, "c": out, "M": M, "N": N}, c["meta"], axis=1, lo=lo, hi=hi,
                              grid=grid_)
    assert cuda_rt.native_launches == before + 2, ck.plan.native.last_reason
    assert torch.equal(out, full)
    np.testing.assert_allclose(full.view(M, N).double().cpu().numpy()[:2],
                               (a.view(M, K)[:2].double() @ b.view(K, N).double()).cpu().numpy(), rtol=1e-4,
                               atol=1e-4)
