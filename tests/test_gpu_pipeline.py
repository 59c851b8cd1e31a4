"""GPU: elementwise kernels on page-locked host tensors take the chunked copy/compute/copy
pipeline (three streams); results equal the CPU oracle bit for bit, host elements the kernel
does not write stay untouched, and in-place (read + write of one array) works."""

import numpy as np
import pytest

import eas
from eas import mk
from oracle.interp import execute

pytestmark = pytest.mark.gpu


@eas.kernel
def add_kernel(a, b, c, N, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


@eas.kernel
def scale_thread(x, y, N, s, BLOCK: eas.constexpr):
    i = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    mk.store(y, i, mk.load(x, i, i < N) * s, i < N)


def _pinned(arr):
    import torch

    t = torch.from_numpy(arr).pin_memory()
    return t


@pytest.fixture
def small_pipeline(monkeypatch, cuda_rt):
    monkeypatch.setenv("EAS_PIPELINE_MIN_BYTES", "1")
    monkeypatch.setattr(type(cuda_rt), "PIPELINE_CHUNK_ELEMS", 1 << 16)
    return cuda_rt


def test_pipelined_add_matches_oracle(small_pipeline):
    import torch

    rng = np.random.default_rng(0)
    n = (1 << 20) + 37
    a, b = (rng.standard_normal(n, dtype=np.float32) for _ in range(2))
    ta, tb = _pinned(a), _pinned(b)
    tc = torch.full((n + 100,), 5.0).pin_memory()  # longer than N: the tail must stay untouched
    launches = small_pipeline.launch_count
    add_kernel(ta, tb, tc, n, BLOCK=1024)
    assert small_pipeline.launch_count - launches > 4  # went through several chunks
    ref = np.zeros(n, np.float32)
    ck = add_kernel.compile(a, b, ref, n, BLOCK=1024)
    execute(ck.ir, {"a": a, "b": b, "c": ref, "N": n})
    np.testing.assert_array_equal(tc.numpy()[:n], ref)
    assert (tc.numpy()[n:] == 5.0).all()


def test_pipelined_in_place(small_pipeline):
    rng = np.random.default_rng(1)
    n = 300_001
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    ta, tb = _pinned(a.copy()), _pinned(b)
    add_kernel(ta, tb, ta, n, BLOCK=256)
    np.testing.assert_array_equal(ta.numpy(), a + b)


def test_pipelined_thread_mode_f16(small_pipeline):
    import torch

    rng = np.random.default_rng(2)
    n = 200_003
    x = rng.standard_normal(n).astype(np.float16)
    tx = _pinned(x)
    ty = torch.zeros(n, dtype=torch.float16).pin_memory()
    scale_thread(tx, ty, n, np.float16(0.5), BLOCK=128)
    np.testing.assert_array_equal(ty.numpy(), (x.astype(np.float32) * np.float32(0.5)).astype(np.float16))


def test_pageable_numpy_takes_the_plain_path(small_pipeline):
    n = 100_000
    a = np.ones(n, np.float32)
    c = np.zeros(n, np.float32)
    launches = small_pipeline.launch_count
    add_kernel(a, a, c, n, BLOCK=1024)
    assert small_pipeline.launch_count - launches == 1
    assert (c == 2).all()
