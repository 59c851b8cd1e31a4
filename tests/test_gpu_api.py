"""GPU: the public API around the kernels — eas.Tensor on cuda, DLPack/torch zero copy,
async launches with the in-flight bound, benchmark(), autotune on the real runtime, and
host-side fault injection leaving the runtime usable."""

import numpy as np
import pytest

import eas
from eas import mk
from easy_as_b200.runtime import cuda_ext

pytestmark = pytest.mark.gpu


@eas.kernel
def add_kernel(a, b, c, N, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


def test_eas_tensor_roundtrip_and_kernel(cuda_rt):
    n = 4099
    a_np = np.random.default_rng(0).standard_normal(n, dtype=np.float32)
    b_np = np.random.default_rng(1).standard_normal(n, dtype=np.float32)
    a = eas.tensor(a_np, device="cuda")
    b = eas.tensor(b_np, device="cuda")
    c = eas.empty_like(a)
    assert c.device == "cuda" and c.__dlpack_device__() == (2, 0)
    add_kernel(a, b, c, n, BLOCK=256)
    np.testing.assert_array_equal(c.numpy(), a_np + b_np)
    np.testing.assert_array_equal(c.to("cpu").numpy(), a_np + b_np)
    f16 = eas.tensor(a_np, device="cuda", dtype=np.float16)
    assert f16.dtype == np.float16
    np.testing.assert_array_equal(f16.numpy(), a_np.astype(np.float16))


def test_dlpack_zero_copy_both_ways(cuda_rt):
    import torch

    t = torch.arange(1000, device="cuda", dtype=torch.float32)
    e = eas.from_dlpack(t, device="cuda")
    assert e._cuda_ptr() == t.data_ptr()
    back = torch.from_dlpack(e)
    assert back.data_ptr() == t.data_ptr()
    back.add_(1.0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(e.numpy(), np.arange(1000, dtype=np.float32) + 1)
    cap = eas.to_dlpack(e)
    assert type(cap).__name__ == "PyCapsule"
    t2 = torch.utils.dlpack.from_dlpack(cap)
    assert t2.data_ptr() == t.data_ptr()
    # import through a raw capsule (not a torch object)
    e2 = eas.from_dlpack(torch.utils.dlpack.to_dlpack(t), device="cuda")
    assert e2._cuda_ptr() == t.data_ptr() and e2.shape == (1000,)


def test_torch_cuda_tensors_on_current_stream(cuda_rt):
    import torch

    n = 1 << 20
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = torch.randn(n, device="cuda")
        b = torch.randn(n, device="cuda")
        c = torch.empty_like(a)
        add_kernel(a, b, c, n, BLOCK=1024, _sync=False)  # ordered after randn on stream s
        d = c * 2
    cuda_rt.synchronize()
    s.synchronize()
    assert torch.equal(d, (a + b) * 2)


def test_async_in_flight_bound(cuda_rt, monkeypatch):
    import torch

    monkeypatch.setattr(cuda_rt, "_max_in_flight", 4)
    n = 1 << 16
    a = torch.randn(n, device="cuda")
    b = torch.randn(n, device="cuda")
    c = torch.empty_like(a)
    for _ in range(20):
        add_kernel(a, b, c, n, BLOCK=1024, _sync=False)
        assert cuda_rt.in_flight() <= 4
    cuda_rt.synchronize()
    assert cuda_rt.in_flight() == 0
    assert torch.equal(c, a + b)


def test_benchmark_returns_seconds(cuda_rt):
    import torch

    n = 1 << 22
    a = torch.randn(n, device="cuda")
    b = torch.randn(n, device="cuda")
    c = torch.empty_like(a)
    ck = add_kernel.compile(a, b, c, n, BLOCK=1024)
    t = cuda_rt.benchmark(ck, {"a": a, "b": b, "c": c, "N": n}, {"BLOCK": 1024}, repeat=5, warmup=2)
    assert 1e-6 < t < 1e-1
    with pytest.raises(ValueError):
        cuda_rt.benchmark(ck, {"a": a.cpu().numpy(), "b": b, "c": c, "N": n}, {"BLOCK": 1024}, repeat=1)


@eas.autotune(configs=[eas.Config(meta={"BLOCK": 256}), eas.Config(meta={"BLOCK": 1024})], key=["N"], warmup=1,
              repeat=3)
@eas.kernel
def add_tuned(a, b, c, N, BLOCK: eas.constexpr = 256):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


def test_autotune_on_device(cuda_rt):
    import torch

    n = 1 << 20 | 5
    a = torch.randn(n, device="cuda")
    b = torch.randn(n, device="cuda")
    c = torch.empty_like(a)
    add_tuned(a, b, c, n)
    assert len(add_tuned._tuned_cache) == 1
    assert torch.equal(c, a + b)


def test_tptg_mismatch_raises(cuda_rt):
    out = np.zeros(10, np.float32)
    with pytest.raises(ValueError):
        add_kernel(out, out, out, 10, BLOCK=256, _tptg=(256, 1, 1))  # spmd expects (1, 1, 1)


def test_injected_launch_failure_then_recovery(cuda_rt):
    import torch

    lib = cuda_ext.load()
    n = 4096
    a = torch.randn(n, device="cuda")
    b = torch.randn(n, device="cuda")
    c = torch.zeros_like(a)
    add_kernel(a, b, c, n, BLOCK=256)  # compiled and loaded
    assert lib.eas_fault_inject(b"launch", 1) == 0
    with pytest.raises(RuntimeError, match="injected"):
        add_kernel(a, b, c, n, BLOCK=256)
    add_kernel(a, b, c, n, BLOCK=256)
    assert torch.equal(c, a + b)


def test_compile_error_is_runtime_error(cuda_rt):
    with pytest.raises(RuntimeError, match="CUDA compile failed"):
        cuda_rt.compile_cubin('extern "C" __global__ void k() { nope; }', "k")


def test_dlpack_export_orders_consumer_stream_without_host_sync(cuda_rt, monkeypatch):
    import torch

    monkeypatch.setattr(cuda_rt, "_max_in_flight", 1 << 20)
    n = 1 << 22
    a = eas.tensor(np.ones(n, np.float32), device="cuda")
    b = eas.tensor(np.full(n, 2.0, np.float32), device="cuda")
    c = eas.empty_like(a)
    for _ in range(20):
        add_kernel(a, b, c, n, BLOCK=1024, _sync=False)  # queued on the legacy default stream
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        t = torch.from_dlpack(c)  # torch passes stream s; eas makes it wait on the device
        assert cuda_rt.in_flight() > 0  # no host synchronisation happened
        d = t * 2
    s.synchronize()
    assert torch.equal(d, torch.full((n,), 6.0, device="cuda"))
    cuda_rt.synchronize()


@pytest.mark.parametrize("kind", ["numpy", "bytearray"])
def test_device_buffer_copy_roundtrip(cuda_rt, kind):
    """Host -> device -> host through a device buffer (reference tests/test_metal_copy.py:21-41)."""
    from easy_as_b200.runtime.cuda import DeviceBuffer

    if kind == "numpy":
        src = np.random.default_rng(1).standard_normal(4096 + 7).astype(np.float32)
        dst = np.empty_like(src)
    else:
        src = bytearray((i * 7 + 3) & 0xFF for i in range(8192))
        dst = bytearray(len(src))
    buf = DeviceBuffer(len(memoryview(src).cast("B")), 0)
    buf.copy_from_host(src)
    buf.copy_to_host(dst)
    buf.free()
    if kind == "numpy":
        assert np.array_equal(dst, src)
    else:
        assert dst == src
