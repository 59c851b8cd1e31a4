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
