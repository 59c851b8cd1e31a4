"""GPU: kernel launches captured in a CUDA graph (torch.cuda.graph) replay correctly."""

import pytest

import eas
from eas import mk

pytestmark = pytest.mark.gpu


@eas.kernel
def axpy(x, y, N, alpha, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(y, offs, mk.fma(mk.load(x, offs, m), alpha, mk.load(y, offs, m)), m)


def test_graph_capture_and_replay(cuda_rt):
    import torch

    n = 1 << 20
    x = torch.randn(n, device="cuda")
    y = torch.zeros(n, device="cuda")
    axpy(x, y, n, 1.0, BLOCK=1024)  # compile + load before capture
    y.zero_()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(3):
            axpy(x, y, n, 1.0, BLOCK=1024, _sync=False)
    assert cuda_rt.in_flight() == 0
    y.zero_()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert torch.allclose(y, 6 * x, rtol=0, atol=1e-5 * x.abs().max().item() * 6)


def test_native_gemms_capture_and_replay(cuda_rt):
    """The tcgen05 (f16 dot GEMM), FFMA (tiled fp32) and mma (f16 staging + tcgen05) native paths
    inside a CUDA graph: replays give the eager results."""
    import torch

    import goldens
    from easy_as_b200.compiler import compile_ir
    from examples.matmul_dot_f16 import grid, matmul_dot_f16

    g = torch.Generator(device="cuda").manual_seed(0)
    M, N, K = 256, 512, 192
    a16 = (torch.randn(M * K, device="cuda", generator=g) / K ** 0.5).half()
    b16 = (torch.randn(K * N, device="cuda", generator=g) / K ** 0.5).half()
    c16 = torch.zeros(M * N, device="cuda")
    tiled = goldens.case("matmul_tiled_c3_full")
    ck_t = compile_ir(goldens.ir_from_json(tiled["opt"]))
    Mt = Nt = 256
    at = torch.randn(Mt * 2048, device="cuda", generator=g)
    bt = torch.randn(2048 * Nt, device="cuda", generator=g)
    ct = torch.zeros(Mt * Nt, device="cuda")
    mma = goldens.case("matmul_simdgroup_512")
    ck_m = compile_ir(goldens.ir_from_json(mma["opt"]))
    am = torch.randn(512 * 512, device="cuda", generator=g)
    bm = torch.randn(512 * 512, device="cuda", generator=g)
    cm = torch.zeros(512 * 512, device="cuda")

    def launch(sync):
        matmul_dot_f16(a16, b16, c16, M, N, K, _grid=grid(1), _sync=sync)
        cuda_rt.run(ck_t, {"a": at, "b": bt, "c": ct, "M": Mt, "N": Nt}, tiled["meta"], sync=sync,
                    grid=(Nt // 32, Mt // 32, 1))
        cuda_rt.run(ck_m, {"a": am, "b": bm, "c": cm, "M": 512, "N": 512}, mma["meta"], sync=sync,
                    grid=tuple(mma["launch"]["grid"]))

    before = cuda_rt.native_launches
    launch(True)                                   # eager: compile, prove, allocate staging
    assert cuda_rt.native_launches == before + 3
    eager = [c16.clone(), ct.clone(), cm.clone()]
    for t in (c16, ct, cm):
        t.zero_()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch(False)
    assert cuda_rt.native_launches == before + 6    # the captured launches took the native paths too
    for t in (c16, ct, cm):
        t.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for got, want in zip((c16, ct, cm), eager):
        assert torch.equal(got, want)
