"""GPU: CUBINs from the on-disk cache (``EAS_CACHE_DIR``) run correctly in a fresh process.

The reference keeps compiled pipelines in memory only (easy_as ``eas/runtime/metal.py:122-132``);
this runtime also stores each NVRTC CUBIN under ``EAS_CACHE_DIR``.  A first process compiles and
stores; a second, fresh process with every NVRTC compile made to fail (host-side fault injection,
``eas_fault_inject("compile", 1)``) must load the same kernels from disk and give results equal to
the CPU oracle's: bit for bit for the add and the row-index fill, and for the fp16 dot kernel on
its generic (non-native) path, whose ordered fma chains the oracle restates exactly."""

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
import numpy as np
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/tests"]
import eas
from eas import mk
from easy_as_b200.runtime import cuda_ext
from oracle.interp import execute
from examples.matmul_dot_f16 import matmul_dot_f16

if sys.argv[2] == "from_disk":
    cuda_ext.load().eas_fault_inject(b"compile", 1)   # any NVRTC compile in this process now fails

@eas.kernel
def add_kernel(a, b, c, N, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)

@eas.kernel
def rows_kernel(out, H, W, BLOCK: eas.constexpr):
    col = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    row = mk.program_id(1)
    mk.store(out, row * W + col, mk.to_f32(row * W + col), (row < H) & (col < W))

rng = np.random.default_rng(0)
n = 1031
a = rng.standard_normal(n, dtype=np.float32); b = rng.standard_normal(n, dtype=np.float32)
c = np.zeros_like(a); want = np.zeros_like(a)
add_kernel(a, b, c, n, BLOCK=256)
execute(add_kernel.compile(a, b, want, n, BLOCK=256).ir, {"a": a, "b": b, "c": want, "N": n})
assert np.array_equal(c, want), "add differs from the oracle"

H, W = 37, 300
out = np.full(H * W, -1.0, np.float32); want = np.full(H * W, -1.0, np.float32)
rows_kernel(out, H, W, BLOCK=128, _grid=(3, H, 1))
execute(rows_kernel.compile(out, H, W, BLOCK=128).ir, {"out": want, "H": H, "W": W}, grid=(3, H, 1))
assert np.array_equal(out, want), "row fill differs from the oracle"

import os
os.environ["EAS_DISABLE_NATIVE"] = "1"      # the generated kernel, not the tcgen05 one
M, N, K = 33, 70, 45
a16 = (rng.standard_normal(M * K) / np.sqrt(K)).astype(np.float16)
b16 = (rng.standard_normal(K * N) / np.sqrt(K)).astype(np.float16)
got = np.zeros(M * N, np.float32); want = np.zeros(M * N, np.float32)
matmul_dot_f16(a16, b16, got, M, N, K, BLOCK_N=128, _grid=(1, M, 1))
execute(matmul_dot_f16.compile(a16, b16, want, M, N, K, BLOCK_N=128).ir,
        {"a": a16, "b": b16, "c": want, "M": M, "N": N, "K": K}, grid=(1, M, 1))
assert np.array_equal(got, want), "dot kernel differs from the oracle"
print("CHILD_OK")
'''


def _run(mode: str, cache: Path) -> subprocess.CompletedProcess:
    env = dict(os.environ, EAS_CACHE_DIR=str(cache), EAS_AUTOTUNE_CACHE="0")
    env.pop("EAS_DISABLE_NATIVE", None)
    return subprocess.run([sys.executable, "-c", CHILD, str(ROOT), mode], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=600)


def test_cubins_from_disk_match_the_oracle_in_a_fresh_process(cuda_rt, tmp_path):
    cache = tmp_path / "cache"
    first = _run("compile", cache)
    assert first.returncode == 0 and "CHILD_OK" in first.stdout, first.stdout[-2000:] + first.stderr[-2000:]
    cubins = sorted(cache.glob("*.cubin"))
    assert len(cubins) >= 3, cubins
    second = _run("from_disk", cache)
    assert second.returncode == 0 and "CHILD_OK" in second.stdout, second.stdout[-2000:] + second.stderr[-2000:]
    # the injected compile failure is armed: without the cache the second process fails
    empty = tmp_path / "empty"
    third = _run("from_disk", empty)
    assert third.returncode != 0 and "CHILD_OK" not in third.stdout
