"""GPU: 256 x 512 CTA-pair tiles (NH = 2) on ragged shapes.

The launcher takes wide tiles only where they add no tile rounds, which the suite's small
shapes never do, so this test forces them (EAS_GEMM_WIDE=1, read once per process) in a child
process.  N a multiple of 8 (16-byte rows, as TMA needs) but not of 512, M not a multiple of 256, batches, both B layouts, and K
tails are held to the same normwise bound as the 256 x 256 tiles."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

CHILD = r'''
import sys
sys.path.insert(0, ".")
import ctypes
import torch
from easy_as_b200.runtime import cuda_ext
from examples.matmul_dot_f16 import grid, matmul_dot_f16

lib = cuda_ext.load()
fails = []
from easy_as_b200.runtime import get_runtime
rt = get_runtime()
# N a multiple of 8 (16-byte f16 rows, as TMA needs) but not of 512
for batch, M, N, K in [(1, 300, 704, 136), (2, 512, 1024, 200), (1, 257, 520, 72), (3, 1000, 1544, 520)]:
    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    before = rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=256,
                   _grid=grid(batch), _sync=True)
    vals = [ctypes.c_int() for _ in range(6)]
    lib.eas_gemm_last_config(*(ctypes.byref(x) for x in vals))
    tn = vals[1].value
    ref = torch.bmm(a.double(), b.double())
    err = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    if rt.native_launches != before + 1 or tn != 512 or not err <= 1e-5 or torch.isnan(c).any():
        fails.append((batch, M, N, K, rt.native_launches - before, tn, err))
    # K-major B through the C entry point
    bt = b.transpose(1, 2).contiguous()
    c2 = torch.full((batch, M, N), float("nan"), device="cuda")
    rc = lib.eas_gemm_f16(a.data_ptr(), bt.data_ptr(), c2.data_ptr(), M, N, K, batch, K, M * K, K, N * K, 1, N, M * N,
                          256, None)
    torch.cuda.synchronize()
    err2 = ((c2.double() - ref).abs().max() / ref.abs().max()).item()
    lib.eas_gemm_last_config(*(ctypes.byref(x) for x in vals))
    if rc != 0 or vals[1].value != 512 or not err2 <= 1e-5:
        fails.append(("kmajor", batch, M, N, K, rc, vals[1].value, err2))
print("FAILS", fails)
sys.exit(1 if fails else 0)
'''


def test_wide_tiles_on_ragged_shapes(cuda_rt):
    env = dict(os.environ, EAS_GEMM_WIDE="1")
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
