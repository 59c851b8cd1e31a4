"""GPU: host outputs of proven GEMM launches.  A host array the kernel only writes is not copied to
the device when the launch provably stores every element of it (the output rectangle of every
batch covers the whole buffer); otherwise it is copied in, so elements the kernel leaves alone
keep their host values.  Arrays here are large enough (> 4 MiB in all) for per-array staging."""

from __future__ import annotations

import numpy as np
import pytest

from examples.matmul_dot_f16 import grid, matmul_dot_f16

pytestmark = pytest.mark.gpu


def _inputs(batch, M, N, K, seed=0):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal(batch * M * K) / np.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal(batch * K * N) / np.sqrt(K)).astype(np.float16)
    return a, b


def _ref(a, b, batch, M, N, K):
    return np.matmul(a.reshape(batch, M, K).astype(np.float64), b.reshape(batch, K, N).astype(np.float64))


def test_fully_stored_output_is_not_copied_in(cuda_rt):
    batch, M, N, K = 2, 512, 1024, 256
    a, b = _inputs(batch, M, N, K)
    c = np.full(batch * M * N, np.nan, np.float32)
    before = cuda_rt.skipped_copy_bytes
    matmul_dot_f16(a, b, c, M, N, K, BLOCK_N=256, _grid=grid(batch))
    assert cuda_rt.skipped_copy_bytes - before == c.nbytes
    ref = _ref(a, b, batch, M, N, K)
    assert not np.isnan(c).any()
    assert np.abs(c.reshape(batch, M, N) - ref).max() <= 1e-5 * np.abs(ref).max()


def test_partly_stored_outputs_keep_their_other_elements(cuda_rt):
    batch, M, N, K = 1, 512, 1024, 256
    a, b = _inputs(batch, M, N, K, seed=1)
    # a larger C buffer: elements past M*N are never stored
    c = np.full(M * N + 4096, 7.0, np.float32)
    before = cuda_rt.skipped_copy_bytes
    matmul_dot_f16(a, b, c, M, N, K, BLOCK_N=256, _grid=grid(batch))
    assert cuda_rt.skipped_copy_bytes == before
    assert np.all(c[M * N:] == 7.0)
    # a grid over the first 300 rows only: rows 300.. keep their values
    c2 = np.full(M * N, 5.0, np.float32)
    matmul_dot_f16(a, b, c2, M, N, K, BLOCK_N=256, _grid=(N // 256, 300, 1))
    assert cuda_rt.skipped_copy_bytes == before
    assert np.all(c2.reshape(M, N)[300:] == 5.0)
    ref = _ref(a, b, 1, M, N, K)[0]
    assert np.abs(c2.reshape(M, N)[:300] - ref[:300]).max() <= 1e-5 * np.abs(ref).max()


def test_batched_gemm_on_pinned_host_tensors_is_pipelined(cuda_rt, monkeypatch):
    """Page-locked host tensors of a batched GEMM: batch slices are copied in, multiplied and copied
    out on three overlapping streams (forced here into many slices); the result is the GEMM's."""
    import torch

    from easy_as_b200.runtime.cuda import CudaRuntime

    monkeypatch.setattr(CudaRuntime, "GEMM_PIPELINE_SLICE_BYTES", 3 << 20)
    batch, M, N, K = 8, 512, 768, 520
    g = torch.Generator().manual_seed(4)
    a = (torch.randn(batch, M, K, generator=g) / K ** 0.5).half().pin_memory()
    b = (torch.randn(batch, K, N, generator=g) / K ** 0.5).half().pin_memory()
    c = torch.full((batch, M, N), float("nan")).pin_memory()
    ck = matmul_dot_f16.compile(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K)
    assert cuda_rt._gemm_pipeline_plan(ck, {"a": a.reshape(-1), "b": b.reshape(-1), "c": c.reshape(-1),
                                            "M": M, "N": N, "K": K}, ((N // 256 + (N % 256 > 0), M, batch),
                                                                      0xFFFFFFFF)) is not None
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, BLOCK_N=256,
                   _grid=grid(batch))
    assert cuda_rt.native_launches - before >= 2           # one native launch per slice
    ref = torch.bmm(a.double(), b.double())
    assert not torch.isnan(c).any()
    assert ((c.double() - ref).abs().max() / ref.abs().max()).item() <= 1e-5
