"""GPU: the tiled matmul family of tests/tiled_variants.py (this repository's own DSL kernels, other
tile shapes, K-tile depths, thread counts and paddings than the reference's) runs natively with the
same bits as the generated kernels."""

import numpy as np
import pytest

from tiled_variants import VARIANTS, grid, tile_mm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("v", VARIANTS, ids=[f"TM{v[0]}_TN{v[1]}_TK{v[2]}_NT{v[3]}_P{v[4]}" for v in VARIANTS])
@pytest.mark.parametrize("M,N,K", [(70, 150, 48), (33, 200, 40)])
def test_variant_native_equals_generated(cuda_rt, monkeypatch, v, M, N, K):
    import torch

    tm, tn, tk, nt, pad = v
    g = torch.Generator(device="cuda").manual_seed(M + K)
    a = torch.randn(M * K, device="cuda", generator=g)
    b = torch.randn(K * N, device="cuda", generator=g)
    outs = []
    for disable in ("0", "1"):
        monkeypatch.setenv("EAS_DISABLE_NATIVE", disable)
        c = torch.full((M * N,), float("nan"), device="cuda")
        before = cuda_rt.native_launches
        tile_mm(a, b, c, M, N, K=K, TM=tm, TN=tn, TK=tk, NT=nt, PAD=pad, _grid=grid(M, N, tm, tn), _sync=True)
        assert (cuda_rt.native_launches == before + 1) == (disable == "0")
        outs.append(c)
    assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32))
    ref = a.view(M, K).double() @ b.view(K, N).double()
    np.testing.assert_allclose(outs[0].view(M, N).double().cpu().numpy(), ref.cpu().numpy(), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("batch,M,N,K", [(5, 70, 150, 64), (3, 128, 96, 32)])
def test_batched_variant_native_equals_generated(cuda_rt, monkeypatch, batch, M, N, K):
    import torch

    from tiled_variants import tile_mm_batched

    tm, tn, tk, nt = 32, 32, 16, 128
    g = torch.Generator(device="cuda").manual_seed(batch)
    a = torch.randn(batch * M * K, device="cuda", generator=g)
    b = torch.randn(batch * K * N, device="cuda", generator=g)
    outs = []
    for disable in ("0", "1"):
        monkeypatch.setenv("EAS_DISABLE_NATIVE", disable)
        c = torch.full((batch * M * N,), float("nan"), device="cuda")
        before = cuda_rt.native_launches
        tile_mm_batched(a, b, c, M, N, K=K, TM=tm, TN=tn, TK=tk, NT=nt,
                        _grid=(-(-N // tn), -(-M // tm), batch), _sync=True)
        assert (cuda_rt.native_launches == before + 1) == (disable == "0")
        outs.append(c)
    assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32))
    ref = torch.bmm(a.view(batch, M, K).double(), b.view(batch, K, N).double())
    np.testing.assert_allclose(outs[0].view(batch, M, N).double().cpu().numpy(), ref.cpu().numpy(), rtol=1e-4,
                               atol=1e-4)
