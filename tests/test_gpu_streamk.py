"""GPU: stream-K in the CTA-pair GEMM (launches whose data-parallel schedule would leave more than
5 % of the pairs idle in its last round, with at least one tile per pair).

Every pair runs an equal share of all tiles' k-blocks; a tile split between two pairs is finished
by the pair that computed its head (k from 0), which adds the other pair's partial tile, always
in the order head + tail.  Checked here: the launch is stream-K (``eas_gemm_last_config`` reports
ksplit 0), every output against float64 (the fp16-GEMM normwise bound of the other GEMM tests and
rtol 2e-2), identical bits over repeated launches, and the same result as the data-parallel
kernel (``EAS_GEMM_STREAMK=0``, in a child process) to f32 rounding."""

from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest

from examples.matmul_dot_f16 import grid, matmul_dot_f16

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _last():
    from easy_as_b200.runtime import cuda_ext

    vals = [ctypes.c_int() for _ in range(6)]
    cuda_ext.check(cuda_ext.load().eas_gemm_last_config(*(ctypes.byref(v) for v in vals)), "last config")
    return [v.value for v in vals]


def _run(cuda_rt, batch, M, N, K, seed, meta):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, **meta, _grid=grid(batch), _sync=True)
    assert cuda_rt.native_launches == before + 1
    return a, b, c


CASES = [
    # (batch, M, N, K, meta): the C4 shards of 8 and 4 GPUs (library choice: 256 x 256 and 256 x 512
    # tiles), a ragged batched launch, and explicit 256 x 256 pair tiles with two k-blocks per stage
    (1, 1024, 8192, 8192, {}),
    (1, 2048, 8192, 8192, {}),
    (10, 512, 1000, 1000, {"BLOCK_N": 256}),
    (1, 1280, 6000, 3000, {"BLOCK_M": 256, "BLOCK_N": 128, "BLOCK_K": 128}),
]


@pytest.mark.parametrize("batch,M,N,K,meta", CASES)
def test_stream_k_matches_float64_and_repeats_bit_for_bit(cuda_rt, batch, M, N, K, meta):
    import torch

    a, b, c = _run(cuda_rt, batch, M, N, K, seed=M + N, meta=meta)
    assert _last()[3] == 0, "expected a stream-K launch"
    worst = 0.0
    for bi in range(batch):
        ref = a[bi].double() @ b[bi].double()
        got = c[bi].double()
        scale = ref.abs().max().item()
        err = (got - ref).abs()
        assert bool((err <= 2e-2 * ref.abs() + 2e-2 * scale).all())
        worst = max(worst, err.max().item() / scale)
    assert not torch.isnan(c).any()
    assert worst <= max(1e-5, 4e-9 * K), worst
    for _ in range(3):
        _, _, again = _run(cuda_rt, batch, M, N, K, seed=M + N, meta=meta)
        assert torch.equal(c.view(torch.int32), again.view(torch.int32))


CHILD = r"""
import sys, torch
sys.path[:0] = [sys.argv[1]]
import eas
from examples.matmul_dot_f16 import grid, matmul_dot_f16
batch, M, N, K = 1, 1024, 8192, 8192
g = torch.Generator(device="cuda").manual_seed(7)
a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
c = torch.empty(batch, M, N, device="cuda")
matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, _grid=grid(batch), _sync=True)
torch.save(c.cpu(), sys.argv[2])
"""


def test_stream_k_agrees_with_the_data_parallel_kernel(cuda_rt, tmp_path):
    import torch

    out = {}
    for mode in ("1", "0"):
        f = tmp_path / f"c{mode}.pt"
        env = dict(os.environ, EAS_GEMM_STREAMK=mode)
        r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(f)], cwd=ROOT, env=env, capture_output=True,
                           text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        out[mode] = torch.load(f)
    sk, dp = out["1"], out["0"]
    assert (sk - dp).abs().max().item() <= 1e-5 * dp.abs().max().item()
