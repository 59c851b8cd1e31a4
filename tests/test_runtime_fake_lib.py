"""CPU: the runtime's host logic against a fake native library (no GPU).

The reference checks its Metal bridge the same way (tests/test_metal_numpy_bridge.py:85-104): a
fake extension receives the launch and the test inspects what the runtime handed it.  Here the
fake ``libeas_cuda`` keeps "device" memory in host buffers, records every call, and executes a
launch by running the CPU oracle on the kernel's IR over views of that memory.  Checked:
small numpy inputs are packed into one pinned bounce buffer and copied in with one
asynchronous copy, large ones are staged per array, scalars are packed little-endian at their
parameter offsets, only written arrays are copied back, buffers are reused across calls, and
launch errors surface as Python exceptions."""

from __future__ import annotations

import ctypes
import re
import struct

import numpy as np
import pytest

import eas
from eas import mk
from easy_as_b200.codegen.cuda import CHECK_TG_SLOT
from easy_as_b200.ir import DType
from easy_as_b200.runtime import cuda_ext
from oracle.interp import OracleError, execute


@eas.kernel
def add_kernel(a, b, c, N, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


@eas.kernel
def scale_kernel(x, y, N, alpha, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(y, offs, mk.load(x, offs, m) * alpha, m)


class FakeLib:
    """The subset of the C ABI the launch path calls, with host memory standing in for HBM.

    Every device allocation has GUARD bytes in front of it: a launch over program sub-range
    [p0, p1) may pass a pointer moved back by p0 * BLOCK elements (slot buffers holding only that
    range), which then still points into the same allocation."""

    GUARD = 1 << 18

    def __init__(self):
        self.mem: dict[int, ctypes.Array] = {}
        self.calls: list[tuple] = []
        self.kernels: dict[int, object] = {}
        self.fail_launch = False
        self.err = b""

    # memory
    def _find(self, ptr: int) -> tuple[ctypes.Array, int]:
        for pool in (self.mem, getattr(self, "pinned", {})):   # pinned memory is mapped: devices reach it
            for base, buf in pool.items():
                if base <= ptr < base + len(buf):
                    return buf, ptr - base
        raise AssertionError(f"pointer {ptr:#x} is not a fake device allocation")

    def eas_alloc_buffer(self, dev, nbytes, out):
        buf = ctypes.create_string_buffer(self.GUARD + max(int(nbytes), 1))
        addr = ctypes.addressof(buf)
        self.mem[addr] = buf
        out._obj.value = addr + self.GUARD
        self.calls.append(("alloc", int(nbytes)))
        return 0

    def eas_free_buffer(self, ptr):
        self.mem.pop(int(ptr) - self.GUARD, None)
        return 0

    def eas_copy_from_host(self, dst, src, nbytes, stream):
        self._find(int(dst))
        ctypes.memmove(int(dst), int(src), int(nbytes))
        self.calls.append(("h2d", int(nbytes)))
        return 0

    def eas_copy_to_host(self, dst, src, nbytes, stream):
        self._find(int(src))
        ctypes.memmove(int(dst), int(src), int(nbytes))
        self.calls.append(("d2h", int(nbytes)))
        return 0

    def eas_copy_from_host_async(self, dst, src, nbytes, stream):
        self._find(int(dst))
        ctypes.memmove(int(dst), int(src), int(nbytes))
        self.calls.append(("h2d_async", int(nbytes)))
        return 0

    def eas_copy_to_host_async(self, dst, src, nbytes, stream):
        self._find(int(src))
        ctypes.memmove(int(dst), int(src), int(nbytes))
        self.calls.append(("d2h_async", int(nbytes)))
        return 0

    def eas_alloc_pinned(self, nbytes, out):
        buf = ctypes.create_string_buffer(max(int(nbytes), 1))
        self.pinned = getattr(self, "pinned", {})
        self.pinned[ctypes.addressof(buf)] = buf
        out._obj.value = ctypes.addressof(buf)
        self.calls.append(("alloc_pinned", int(nbytes)))
        return 0

    def eas_pinned_device_pointer(self, host, out):
        out._obj.value = int(host)
        return 0

    def eas_free_pinned(self, p):
        getattr(self, "pinned", {}).pop(int(p), None)
        return 0

    # compile / load: the "binary" is the source text; the pipeline handle indexes it
    def eas_versions(self, drv, nvrtc):
        drv._obj.value, nvrtc._obj.value = 12090, 12090
        return 0

    def eas_compile(self, src, name, opts, nopts, img, size):
        self._img = ctypes.create_string_buffer(bytes(src))
        img._obj.value = ctypes.addressof(self._img)
        size._obj.value = len(src)
        return 0

    def eas_free_host(self, p):
        return 0

    def eas_pipeline_load(self, dev, cubin, n, name, smem, out):
        h = len(self.kernels) + 1
        self.kernels[h] = name
        out._obj.value = h
        return 0

    # launch: decode the parameter block with the kernel's layout, run the oracle
    def eas_launch(self, pipe, grid, block, smem, stream, blob, offsets, count):
        self.calls.append(("launch", tuple(grid), tuple(block)))
        if self.fail_launch:
            self.err = b"fake launch failure"
            return cuda_ext.EAS_ERR_LAUNCH
        ck = self.current
        layout = ck.plan.layout
        assert [offsets[i] for i in range(count)] == [o for _p, o, _f in layout.entries]
        args, hidden = {}, {}
        for p, off, fmt in layout.entries:
            (v,) = struct.unpack_from(fmt, blob, off)
            if p.kind == "buffer":
                buf, at = self._find(v)
                arg = next(a for a in ck.ir.args if a.name == p.arg)
                dt = np.float32 if arg.dtype == DType.F32 else np.float16
                args[p.arg] = np.frombuffer(buf, dtype=dt, count=(len(buf) - at) // np.dtype(dt).itemsize,
                                            offset=at)
            elif p.kind in ("hidden", "check"):
                hidden[p.name] = v
            else:
                args[p.arg] = v
        self.scalars = {k: v for k, v in args.items() if not isinstance(v, np.ndarray)}
        self.hidden = hidden
        for p, _off, _fmt in layout.entries:   # a checked kernel's buffers are exactly eas_n_<name> long
            if p.kind == "check" and p.name.startswith("eas_n_"):
                args[p.arg] = args[p.arg][:hidden[p.name]]
        if getattr(self, "violation", None) is not None:   # a checked kernel's device-side record
            buf, at = self._find(hidden["eas_err"])
            np.frombuffer(buf, np.uint32, 4, at)[:3] = (1, *self.violation)
            return 0
        run = dict(grid=tuple(grid), pid_base=(hidden["eas_pid_x"], hidden["eas_pid_y"], hidden["eas_pid_z"]),
                   ntx=hidden["eas_ntx"])
        self.pid_bases = getattr(self, "pid_bases", []) + [run["pid_base"]]
        if "eas_err" not in hidden:
            execute(ck.ir, args, **run)
            return 0
        try:   # a checked kernel: an access the oracle refuses becomes the device's error record
            execute(ck.ir, args, **run)
        except OracleError as e:
            m = re.match(r"out-of-bounds (load from|store to) '?(\w+)'?: index (\d+)", str(e))
            assert m, str(e)
            names = [a.name for a in ck.ir.args]
            slot = names.index(m.group(2)) if m.group(2) in names else CHECK_TG_SLOT
            buf, at = self._find(hidden["eas_err"])
            np.frombuffer(buf, np.uint32, 4, at)[:3] = (1, 2 * slot + (m.group(1) == "store to"), int(m.group(3)))
        return 0

    def eas_launch_pdl(self, *args):
        self.pdl_launches = getattr(self, "pdl_launches", 0) + 1
        return self.eas_launch(*args)

    def eas_pad_f16_2d(self, src, dst, rows, cols_pad, ld_src, ld_dst, rows_valid, cols_valid, batch, bs_src, bs_dst,
                       stream):
        """numpy stand-in for the f16 re-pitching kernel (zero outside the valid extent)."""
        if int(dst) % 16 or cols_pad % 8 or ld_dst % 8:
            return 4
        self.calls.append(("pad_f16", rows, cols_pad, batch))
        for z in range(batch):
            for r in range(rows):
                out = np.zeros(cols_pad, np.float16)
                if r < rows_valid:
                    buf, at = self._find(int(src) + 2 * (z * bs_src + r * ld_src))
                    out[:cols_valid] = np.frombuffer(buf, np.float16, count=cols_valid, offset=at)
                dbuf, dat = self._find(int(dst) + 2 * (z * bs_dst + r * ld_dst))
                ctypes.memmove(ctypes.addressof(dbuf) + dat, out.ctypes.data, 2 * cols_pad)
        return 0

    def eas_gemm_f16_tile(self, a, b, c, M, N, K, batch, lda, a_bs, ldb, b_bs, b_kmajor, ldc, c_bs, tile_m, block_n,
                          block_k, stream):
        """The explicit-tile entry: same sums as eas_gemm_f16 (the tile only changes speed)."""
        if tile_m not in (0, 128, 256) or block_k not in (0, 64, 128):
            return 4
        return self.eas_gemm_f16(a, b, c, M, N, K, batch, lda, a_bs, ldb, b_bs, b_kmajor, ldc, c_bs, block_n, stream)

    def eas_gemm_f16(self, a, b, c, M, N, K, batch, lda, a_bs, ldb, b_bs, b_kmajor, ldc, c_bs, block_n, stream):
        """numpy stand-in for the tcgen05 GEMM over the fake device memory."""
        self.calls.append(("gemm", M, N, K, batch))

        def view(ptr, dt, count):
            buf, at = self._find(int(ptr))
            return np.frombuffer(buf, dtype=dt, count=count, offset=at)

        for z in range(batch):
            A = view(a + 2 * z * a_bs, np.float16, (M - 1) * lda + K).astype(np.float64)
            A = np.lib.stride_tricks.as_strided(A, (M, K), (8 * lda, 8))
            if b_kmajor:
                B = view(b + 2 * z * b_bs, np.float16, (N - 1) * ldb + K).astype(np.float64)
                B = np.lib.stride_tricks.as_strided(B, (N, K), (8 * ldb, 8)).T
            else:
                B = view(b + 2 * z * b_bs, np.float16, (K - 1) * ldb + N).astype(np.float64)
                B = np.lib.stride_tricks.as_strided(B, (K, N), (8 * ldb, 8))
            C = view(c + 4 * z * c_bs, np.float32, (M - 1) * ldc + N)
            out = (A @ B).astype(np.float32)
            for m in range(M):
                C[m * ldc:m * ldc + N] = out[m]
        return 0

    # streams, events, status
    def eas_stream_synchronize(self, stream):
        return 0

    def eas_stream_is_capturing(self, stream, out):
        out._obj.value = int(getattr(self, "capturing", 0))
        return 0

    def eas_gemm_status(self, dev, out):
        out._obj.value = 0
        return 0

    def eas_host_is_pinned(self, ptr, out):
        out._obj.value = int(any(lo <= int(ptr) < hi for lo, hi in getattr(self, "pinned_ranges", [])))
        return 0

    # streams and events: the fake executes every call at once, in order
    def eas_stream_create(self, dev, out):
        self._handles = getattr(self, "_handles", 1000) + 1
        out._obj.value = self._handles
        return 0

    def eas_event_create(self, out):
        return self.eas_stream_create(0, out)

    def eas_event_record(self, ev, stream):
        return 0

    def eas_event_destroy(self, ev):
        return 0

    def eas_stream_wait_event(self, stream, ev):
        return 0

    def eas_is_available(self):
        return 1

    def eas_last_error(self):
        return self.err


@pytest.fixture
def fake(monkeypatch):
    from easy_as_b200.runtime.cuda import CudaRuntime

    lib = FakeLib()
    monkeypatch.setattr(cuda_ext, "_lib", lib)
    monkeypatch.setenv("EAS_CACHE_DIR", "off")
    rt = CudaRuntime()
    rt.default_device = lambda: 0  # type: ignore[method-assign]
    return lib, rt


def _run(lib, rt, kernel, args, grid=None, **meta):
    ck = kernel.compile(*args, **meta)
    lib.current = ck
    names = [a.name for a in ck.ir.args]
    rt.run(ck, dict(zip(names, args)), meta, sync=True, grid=grid)
    return ck


def test_numpy_inputs_are_staged_and_only_outputs_copied_back(fake, monkeypatch):
    """With zero-copy off: one packed copy in, one copy out of the written array."""
    monkeypatch.setenv("EAS_ZERO_COPY", "0")
    lib, rt = fake
    n = 1024 + 7
    rng = np.random.default_rng(0)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    c = np.zeros_like(a)
    _run(lib, rt, add_kernel, (a, b, c, n), BLOCK=256)
    assert np.array_equal(c, a + b)
    kinds = [k[0] for k in lib.calls]
    assert kinds.count("launch") == 1
    assert [k for k in lib.calls if k[0] == "launch"][0][1] == (5, 1, 1)   # ceil(1031 / 256) programs
    # one packed copy in (a, b, c at 256-byte aligned offsets), one copy out of c alone
    assert [k for k in lib.calls if k[0].startswith("h2d")] == [("h2d_async", 3 * 4352)]
    assert [k for k in lib.calls if k[0].startswith("d2h")] == [("d2h_async", c.nbytes)]
    assert lib.scalars == {"N": n}


def test_large_host_arrays_are_staged_per_array(fake):
    lib, rt = fake
    rt.BOUNCE_MAX_BYTES = 1024                     # force the per-array path
    n = 1000
    a = np.arange(n, dtype=np.float32)
    b = np.ones(n, np.float32)
    c = np.zeros(n, np.float32)
    _run(lib, rt, add_kernel, (a, b, c, n), BLOCK=256)
    assert np.array_equal(c, a + b)
    assert sum(1 for k in lib.calls if k[0] == "h2d") == 3
    assert [k for k in lib.calls if k[0].startswith("d2h")] == [("d2h", c.nbytes)]


def test_scalars_are_packed_at_their_offsets(fake):
    lib, rt = fake
    n = 300
    x = np.arange(n, dtype=np.float32)
    y = np.zeros_like(x)
    _run(lib, rt, scale_kernel, (x, y, n, 0.5), BLOCK=128)
    assert lib.scalars == {"N": n, "alpha": 0.5}
    assert np.array_equal(y, x * np.float32(0.5))


def test_staging_buffers_are_pooled(fake):
    lib, rt = fake
    n = 513
    a = np.ones(n, np.float32)
    b = np.ones(n, np.float32)
    c = np.zeros(n, np.float32)
    _run(lib, rt, add_kernel, (a, b, c, n), BLOCK=256)
    allocs = sum(1 for k in lib.calls if k[0].startswith("alloc"))
    _run(lib, rt, add_kernel, (a, b, c, n), BLOCK=256)
    assert sum(1 for k in lib.calls if k[0].startswith("alloc")) == allocs    # second call reuses them
    assert np.array_equal(c, np.full(n, 2.0, np.float32))


def test_same_array_passed_twice_is_staged_once(fake, monkeypatch):
    monkeypatch.setenv("EAS_ZERO_COPY", "0")
    lib, rt = fake
    n = 100
    a = np.arange(n, dtype=np.float32)
    c = np.zeros_like(a)
    _run(lib, rt, add_kernel, (a, a, c, n), BLOCK=64)
    assert [k for k in lib.calls if k[0].startswith("h2d")] == [("h2d_async", 2 * 512)]   # a and c once each
    assert np.array_equal(c, a + a)


def test_launch_error_raises_with_the_library_message(fake):
    lib, rt = fake
    lib.fail_launch = True
    a = np.ones(10, np.float32)
    with pytest.raises(cuda_ext.CudaError, match="fake launch failure"):
        _run(lib, rt, add_kernel, (a, a.copy(), np.zeros(10, np.float32), 10), BLOCK=32)


def test_async_call_with_host_inputs_does_not_share_the_bounce_buffer(fake):
    """A read-only host input with _sync=False is staged in its own buffer (kept alive by the
    launch), never in the bounce buffer the next call refills."""
    lib, rt = fake
    n = 64
    x = np.arange(n, dtype=np.float32)
    y = np.zeros(n, np.float32)
    ck = scale_kernel.compile(x, y, n, 2.0, BLOCK=64)
    lib.current = ck
    import torch

    out = torch.zeros(n)          # CPU tensor: written, so this call still syncs and copies back
    rt.run(ck, {"x": x, "y": out.numpy(), "N": n, "alpha": 2.0}, {"BLOCK": 64}, sync=False)
    assert not any(k[0] == "h2d_async" for k in lib.calls)
    assert np.array_equal(out.numpy(), x * 2)


def test_generated_kernels_launch_with_pdl_by_default(fake, monkeypatch):
    """Generated kernels begin with griddepcontrol.wait, and the runtime launches them with
    programmatic dependent launch unless EAS_PDL=0."""
    lib, rt = fake
    n = 64
    x = np.arange(n, dtype=np.float32)
    y = np.zeros(n, np.float32)
    ck = _run(lib, rt, scale_kernel, (x, y, n, 3.0), BLOCK=64)
    assert "griddepcontrol.wait" in ck.src
    assert getattr(lib, "pdl_launches", 0) == 1
    from easy_as_b200.runtime.cuda import CudaRuntime

    monkeypatch.setenv("EAS_PDL", "0")
    rt2 = CudaRuntime()
    rt2.default_device = lambda: 0
    _run(lib, rt2, scale_kernel, (x, y, n, 3.0), BLOCK=64)
    assert lib.pdl_launches == 1


def test_host_output_stored_in_full_is_not_copied_in(fake):
    """Per-array staging (bounce off): the GEMM's output array is written in full by the launch, so
    its copy-in is skipped; a larger output buffer, which the launch does not cover, is copied in
    and its extra elements come back unchanged."""
    from examples.matmul_dot_f16 import matmul_dot_f16

    lib, rt = fake
    rt.BOUNCE_MAX_BYTES = 0
    M, N, K = 16, 32, 8
    rng = np.random.default_rng(0)
    a = rng.standard_normal(M * K).astype(np.float16)
    b = rng.standard_normal(K * N).astype(np.float16)
    c = np.full(M * N, np.nan, np.float32)
    _run(lib, rt, matmul_dot_f16, (a, b, c, M, N, K), grid=(1, M, 1), BLOCK_N=256)
    h2d = [k[1] for k in lib.calls if k[0] == "h2d"]
    assert sorted(h2d) == sorted([a.nbytes, b.nbytes])          # no copy of c
    assert rt.skipped_copy_bytes == c.nbytes
    ref = a.reshape(M, K).astype(np.float64) @ b.reshape(K, N).astype(np.float64)
    np.testing.assert_allclose(c.reshape(M, N), ref, rtol=1e-5, atol=1e-5)

    lib.calls.clear()
    c2 = np.full(M * N + 8, 3.0, np.float32)
    _run(lib, rt, matmul_dot_f16, (a, b, c2, M, N, K), grid=(1, M, 1), BLOCK_N=256)
    assert sorted(k[1] for k in lib.calls if k[0] == "h2d") == sorted([a.nbytes, b.nbytes, c2.nbytes])
    assert np.all(c2[M * N:] == 3.0)


def test_elementwise_launch_on_host_arrays_is_zero_copy(fake):
    """An elementwise kernel on small host arrays works on the page-locked bounce buffer in place:
    no copies either way; a non-elementwise kernel still copies."""
    lib, rt = fake
    n = 1031
    rng = np.random.default_rng(3)
    a = rng.standard_normal(n, dtype=np.float32)
    b = rng.standard_normal(n, dtype=np.float32)
    c = np.zeros_like(a)
    _run(lib, rt, add_kernel, (a, b, c, n), BLOCK=256)
    assert np.array_equal(c, a + b)
    assert not any(k[0] in ("h2d", "h2d_async", "d2h", "d2h_async") for k in lib.calls)

    from examples.matmul_dot_f16 import matmul_dot_f16

    M, N, K = 8, 16, 8
    x = rng.standard_normal(M * K).astype(np.float16)
    y = rng.standard_normal(K * N).astype(np.float16)
    z = np.zeros(M * N, np.float32)
    lib.calls.clear()
    _run(lib, rt, matmul_dot_f16, (x, y, z, M, N, K), grid=(1, M, 1), BLOCK_N=256)
    assert any(k[0] == "h2d_async" for k in lib.calls) and any(k[0] == "d2h_async" for k in lib.calls)


def test_batched_gemm_on_pinned_host_arrays_is_pipelined(fake, monkeypatch):
    """Page-locked host arrays of a batched GEMM: batch slices are copied in, multiplied (one native
    launch per slice) and copied out; C is never copied in and the result is the GEMM's."""
    from easy_as_b200.runtime.cuda import CudaRuntime
    from examples.matmul_dot_f16 import matmul_dot_f16

    lib, rt = fake
    monkeypatch.setattr(CudaRuntime, "GEMM_PIPELINE_SLICE_BYTES", 2 * 2 * (16 * 8 + 8 * 32))   # two batches of A + B per slice
    batch, M, N, K = 5, 16, 32, 8
    rng = np.random.default_rng(1)
    a = rng.standard_normal(batch * M * K).astype(np.float16)
    b = rng.standard_normal(batch * K * N).astype(np.float16)
    c = np.full(batch * M * N, np.nan, np.float32)
    lib.pinned_ranges = [(x.ctypes.data, x.ctypes.data + x.nbytes) for x in (a, b, c)]
    _run(lib, rt, matmul_dot_f16, (a, b, c, M, N, K), grid=(1, M, batch), BLOCK_N=256)
    gemms = [k for k in lib.calls if k[0] == "gemm"]
    assert [g[4] for g in gemms] == [2, 2, 1]                       # slices of 2, 2 and 1 batches
    copies_in = [k[1] for k in lib.calls if k[0] == "h2d_async"]
    assert sum(copies_in) == a.nbytes + b.nbytes                    # C never copied in
    assert sum(k[1] for k in lib.calls if k[0] == "d2h_async") == c.nbytes
    ref = np.matmul(a.reshape(batch, M, K).astype(np.float64), b.reshape(batch, K, N).astype(np.float64))
    np.testing.assert_allclose(c.reshape(batch, M, N), ref, rtol=1e-5, atol=1e-5)


def test_device_eas_tensors_launch_without_host_copies(fake, monkeypatch):
    """eas.Tensor(device="cuda") arguments are passed by device pointer: no staging, no copies,
    one launch, and the specialisation cache is hit on the second call."""
    import easy_as_b200.runtime as R

    lib, rt = fake
    rt._available = True
    monkeypatch.setattr(R, "_cuda", rt)
    n = 3000
    x = np.arange(n, dtype=np.float32)
    a, b, c = (eas.empty(n, device="cuda", dtype=np.float32) for _ in range(3))
    for t, v in ((a, x), (b, 2 * x)):
        buf, at = lib._find(t._cuda_ptr())
        np.frombuffer(buf, np.float32, n, at)[:] = v
    lib.current = add_kernel.compile(a, b, c, n, BLOCK=1024)
    lib.calls.clear()
    add_kernel(a, b, c, n, BLOCK=1024)
    cached = len(add_kernel._cache)
    add_kernel(a, b, c, n, BLOCK=1024)
    assert [k[0] for k in lib.calls] == ["launch", "launch"]
    buf, at = lib._find(c._cuda_ptr())
    np.testing.assert_array_equal(np.frombuffer(buf, np.float32, n, at), 3 * x)
    assert len(add_kernel._cache) == cached


@pytest.fixture
def checked(monkeypatch):
    monkeypatch.setenv("EAS_BOUNDS_CHECK", "1")


def test_checked_kernel_gets_each_buffers_bounds_and_a_clear_record(fake, checked):
    """EAS_BOUNDS_CHECK=1: the launch carries (lo, n) of every buffer and the error-record pointer;
    the record is cleared before the launch and a clean record raises nothing."""
    lib, rt = fake
    a = np.arange(1031, dtype=np.float32)
    b = np.ones(1031, np.float32)
    c = np.zeros(1031, np.float32)
    ck = _run(lib, rt, add_kernel, (a, b, c, 1031), BLOCK=256)
    assert ck.plan.checked
    h = lib.hidden
    assert (h["eas_lo_a"], h["eas_n_a"], h["eas_lo_b"], h["eas_n_b"], h["eas_lo_c"], h["eas_n_c"]) == \
        (0, 1031, 0, 1031, 0, 1031)
    buf, at = lib._find(h["eas_err"])
    assert not np.frombuffer(buf, np.uint32, 4, at).any()
    np.testing.assert_array_equal(c, a + b)


def test_checked_kernel_raises_on_a_recorded_violation(fake, checked):
    """A record (1, 2 * slot + is_store, index) written by the device raises IndexError naming the
    buffer, the access and its valid range."""
    lib, rt = fake
    a, b, c = np.ones(100, np.float32), np.ones(100, np.float32), np.zeros(100, np.float32)
    lib.violation = (2 * 2 + 1, 130)   # store to argument 2 ("c") at element 130
    with pytest.raises(IndexError, match=r"out-of-bounds store to 'c' at element 130 \(valid elements: \[0, 100\)\)"):
        _run(lib, rt, add_kernel, (a, b, c, 100), BLOCK=256)
    lib.violation = (2 * 1, 7)
    with pytest.raises(IndexError, match=r"load from 'b' at element 7"):
        _run(lib, rt, add_kernel, (a, b, c, 100), BLOCK=256)


def test_checked_kernel_reports_threadgroup_violations(fake, checked):
    """Slots from CHECK_TG_SLOT on name a threadgroup allocation and its size."""
    from easy_as_b200.codegen.cuda import CHECK_TG_SLOT

    @eas.kernel
    def tg_copy(x, y, N, BLOCK: eas.constexpr):
        t = mk.tid(0, BLOCK)
        s = mk.alloc_tg(BLOCK)
        g = mk.program_id(0) * BLOCK + t
        mk.store(s, t, mk.load(x, g, g < N), True)
        mk.barrier()
        mk.store(y, g, mk.load(s, t, True), g < N)

    lib, rt = fake
    x, y = np.arange(64, dtype=np.float32), np.zeros(64, np.float32)
    lib.violation = (2 * CHECK_TG_SLOT + 1, 99)
    with pytest.raises(IndexError, match=r"store to threadgroup allocation #0 at element 99 \(it holds 32 elements\)"):
        _run(lib, rt, tg_copy, (x, y, 64), BLOCK=32)


def test_checked_kernels_run_as_generated(fake, checked):
    """A checked fp16 dot GEMM has no native plan (the generated kernel, with its checks, runs) and
    an elementwise kernel is not offered to the host pipelines."""
    from examples.matmul_dot_f16 import matmul_dot_f16

    lib, rt = fake
    M, N, K = 16, 32, 8
    a = np.ones(M * K, np.float16)
    b = np.ones(K * N, np.float16)
    c = np.zeros(M * N, np.float32)
    ck = matmul_dot_f16.compile(a, b, c, M, N, K, BLOCK_N=256)
    assert ck.plan.checked and ck.plan.native is None
    ck2 = add_kernel.compile(c, c, c, M * N, BLOCK=256)
    assert ck2.plan.checked and ck2.plan.elementwise is None


def test_checked_range_launch_passes_the_element_base(fake, checked, monkeypatch):
    """run_range with buffer_base={name: e}: the buffer holds global elements [e, e + n)."""
    lib, rt = fake
    n = 512
    a, b, c = (eas.empty(n, device="cuda", dtype=np.float32) for _ in range(3))
    ck = add_kernel.compile(a, b, c, 4 * n, BLOCK=256)
    lib.current = ck
    monkeypatch.setattr(lib, "eas_launch", lambda *args: (setattr(lib, "blob", args[5]), 0)[1])
    monkeypatch.setattr(lib, "eas_launch_pdl", lib.eas_launch)
    rt.run_range(ck, {"a": a, "b": b, "c": c, "N": 4 * n}, {"BLOCK": 256}, axis=0, lo=4, hi=6,
                 buffer_base={"a": 1024, "b": 1024, "c": 1024})
    vals = {p.name: struct.unpack_from(f, lib.blob, o)[0] for p, o, f in ck.plan.layout.entries}
    assert (vals["eas_lo_c"], vals["eas_n_c"], vals["eas_pid_x"]) == (1024, n, 4)


def test_checked_kernel_refuses_graph_capture(fake, checked):
    lib, rt = fake
    n = 256
    a, b, c = (eas.empty(n, device="cuda", dtype=np.float32) for _ in range(3))
    ck = add_kernel.compile(a, b, c, n, BLOCK=256)
    lib.current = ck
    lib.capturing = 1
    with pytest.raises(ValueError, match="cannot be captured"):
        rt.run(ck, {"a": a, "b": b, "c": c, "N": n}, {"BLOCK": 256}, sync=False, grid=None)


def test_out_of_bounds_corpus_raises_index_error_when_checked(fake, checked):
    """Each kernel of tests/oob_kernels.py, launched checked: the (simulated) device record reaches
    the caller as IndexError naming the buffer and the access."""
    from oob_kernels import OOB_CASES

    lib, rt = fake
    for _cid, kernel, make, meta, grid, buf, kind in OOB_CASES:
        verb = "load from" if kind == "load" else "store to"
        where = f"{buf!r}" if buf else "threadgroup allocation #0"
        with pytest.raises(IndexError, match=f"out-of-bounds {verb} {where}"):
            _run(lib, rt, kernel, make(), grid=grid, **meta)


def test_elementwise_launch_on_pinned_host_arrays_is_pipelined(fake, monkeypatch):
    """Large page-locked host arrays of an elementwise kernel: program ranges of one chunk each are
    copied in, run on slot buffers (pointers moved back by the chunk start, program ids offset by
    it) and copied out.  c is only written, so it is never copied in, and only its elements below
    the store bound N come back: host elements past N keep their values."""
    from easy_as_b200.runtime.cuda import CudaRuntime

    lib, rt = fake
    monkeypatch.setenv("EAS_PIPELINE_MIN_BYTES", "4096")
    monkeypatch.setattr(CudaRuntime, "PIPELINE_CHUNK_ELEMS", 1024)
    n, extra = 10_000, 37
    rng = np.random.default_rng(3)
    a = rng.standard_normal(n + extra).astype(np.float32)
    b = rng.standard_normal(n + extra).astype(np.float32)
    c = np.full(n + extra, -7.0, np.float32)
    lib.pinned_ranges = [(x.ctypes.data, x.ctypes.data + x.nbytes) for x in (a, b, c)]
    lib.pid_bases = []
    _run(lib, rt, add_kernel, (a, b, c, n), BLOCK=256)
    gx = -(-n // 256)
    assert lib.pid_bases == [(p0, 0, 0) for p0 in range(0, gx, 4)]
    assert sum(k[1] for k in lib.calls if k[0] == "h2d_async") == 2 * 4 * (n + extra)   # a and b, not c
    assert sum(k[1] for k in lib.calls if k[0] == "d2h_async") == 4 * n
    np.testing.assert_array_equal(c[:n], a[:n] + b[:n])
    assert (c[n:] == -7.0).all()


def test_thread_mode_program_offsets_reach_the_oracle(fake):
    """run_range on a thread-mode kernel: the launch's program-id offset and exact thread count
    decide which global threads run, as in the generated kernel."""

    @eas.kernel
    def tfill(y, N, BLOCK: eas.constexpr):
        t = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
        mk.store(y, t, mk.to_f32(t) + 0.5, t < N)

    lib, rt = fake
    n = 1000
    y = eas.empty(n, device="cuda", dtype=np.float32)
    buf, at = lib._find(y._cuda_ptr())
    view = np.frombuffer(buf, np.float32, n, at)
    view[:] = -1.0
    ck = tfill.compile(y, n, BLOCK=128)
    lib.current = ck
    rt.run_range(ck, {"y": y, "N": n}, {"BLOCK": 128}, axis=0, lo=3, hi=8)
    want = np.full(n, -1.0, np.float32)
    want[3 * 128:n] = np.arange(3 * 128, n, dtype=np.float32) + 0.5
    np.testing.assert_array_equal(view, want)


def test_program_id_shards_on_slice_buffers(fake, monkeypatch):
    """shard.run_shard for each of three ranks, each holding only its element slice of a, b and c
    (buffer_base = the slice start): the slices put together equal a + b.  The ranks run one
    after another in this process; no collective is involved."""
    import easy_as_b200.runtime as R
    from easy_as_b200.shard import element_range, run_shard

    lib, rt = fake
    rt._available = True
    monkeypatch.setattr(R, "_cuda", rt)
    n, world, block = 30_001, 3, 256
    rng = np.random.default_rng(5)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    out = np.zeros(n, np.float32)
    for rank in range(world):
        e0, e1 = element_range(n, block, rank, world)
        sl = {}
        for name, src in (("a", a), ("b", b), ("c", None)):
            t = eas.empty(e1 - e0, device="cuda", dtype=np.float32)
            if src is not None:
                buf, at = lib._find(t._cuda_ptr())
                np.frombuffer(buf, np.float32, e1 - e0, at)[:] = src[e0:e1]
            sl[name] = t
        lib.current = add_kernel.compile(sl["a"], sl["b"], sl["c"], n, BLOCK=block)
        lo, hi = run_shard(add_kernel, sl["a"], sl["b"], sl["c"], n, BLOCK=block, _rank=rank, _world=world,
                           _buffer_base={"a": e0, "b": e0, "c": e0})
        assert (lo * block, min(hi * block, n)) == (e0, e1)
        buf, at = lib._find(sl["c"]._cuda_ptr())
        out[e0:e1] = np.frombuffer(buf, np.float32, e1 - e0, at)
    np.testing.assert_array_equal(out, a + b)


# -- prepared repeated launches (Kernel.__call__ fast path) -------------------------------------


@pytest.fixture
def fast(fake, monkeypatch):
    """The fake runtime as the process runtime, so kernel calls reach it."""
    import easy_as_b200.runtime as runtime_mod

    lib, rt = fake
    rt._available = True
    monkeypatch.setattr(runtime_mod, "_cuda", rt)
    lib.eas_event_create = lambda p: (setattr(p._obj, "value", 4096), 0)[1]
    lib.eas_event_record = lambda ev, s: 0
    lib.eas_event_synchronize = lambda ev: 0
    lib.eas_stream_is_capturing = lambda s, p: 0
    lib.eas_set_device = lambda d: 0
    return lib, rt


@eas.kernel
def axpy_kernel(x, y, out, N, alpha, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(out, offs, mk.load(x, offs, m) * alpha + mk.load(y, offs, m), m)


def test_repeated_device_calls_take_the_prepared_launch(fast):
    """Device buffers: the second and later identical calls make one launch each without
    re-resolving their arguments, with the buffer pointers of each call patched in."""
    lib, rt = fast
    n = 1000
    k = eas.kernel(axpy_kernel.fn)
    xs = [eas.tensor(np.random.default_rng(i).standard_normal(n).astype(np.float32), device="cuda") for i in range(3)]
    y = eas.tensor(np.ones(n, np.float32), device="cuda")
    out = eas.empty_like(y)
    lib.current = k.compile(xs[0], y, out, n, 2.0, BLOCK=256)
    calls = []
    orig_resolve = rt._resolve
    rt._resolve = lambda *a, **kw: (calls.append(1), orig_resolve(*a, **kw))[1]

    def want(x, alpha):
        w = np.zeros(n, np.float32)
        execute(lib.current.ir, {"x": x.numpy(), "y": y.numpy(), "out": w, "N": n, "alpha": alpha})
        return w

    for x in xs:
        k(x, y, out, n, 2.0, BLOCK=256, _sync=False)
        rt.synchronize()
        np.testing.assert_array_equal(out.numpy(), want(x, 2.0))
    assert len(calls) == 1 and len(k._fast) == 1
    # a different scalar is a different prepared launch; its result uses the new value
    k(xs[0], y, out, n, 3.0, BLOCK=256)
    np.testing.assert_array_equal(out.numpy(), want(xs[0], 3.0))
    assert len(k._fast) == 2


def test_repeated_small_host_calls_use_the_bounce_buffer_in_place(fast):
    """Small numpy arrays of an elementwise kernel: each call copies its inputs into the pinned
    buffer, launches on it in place and copies the written array back; arrays passed twice
    (aliases) get their own prepared launch."""
    lib, rt = fast
    n = 1031
    k = eas.kernel(add_kernel.fn)
    rng = np.random.default_rng(0)
    a, b = rng.standard_normal(n, dtype=np.float32), rng.standard_normal(n, dtype=np.float32)
    c = np.zeros(n, np.float32)
    lib.current = k.compile(a, b, c, n, BLOCK=256)
    for i in range(3):
        a = rng.standard_normal(n, dtype=np.float32)
        k(a, b, c, n, BLOCK=256)
        np.testing.assert_array_equal(c, a + b)
    assert len(k._fast) == 1
    k(a, a, a, n, BLOCK=256)          # in place: a = a + a
    assert len(k._fast) == 2


def test_fast_launch_can_be_switched_off(fast, monkeypatch):
    monkeypatch.setenv("EAS_FAST_LAUNCH", "0")
    k = eas.kernel(add_kernel.fn)
    assert k._fast is None


def test_repeated_shard_calls_take_the_prepared_range_launch(fast):
    """run_shard's later identical calls reuse the prepared range launch: the same program range,
    the hidden program-id base and slice pointers moved back by the buffer base."""
    from easy_as_b200.shard import element_range, run_shard

    lib, rt = fast
    n, world, rank = 1 << 15, 4, 2
    k = eas.kernel(add_kernel.fn)
    lo, hi = element_range(n, 256, rank, world)
    base = {"a": lo, "b": lo, "c": lo}
    c = eas.tensor(np.zeros(hi - lo, np.float32), device="cuda")
    b = eas.tensor(np.ones(hi - lo, np.float32), device="cuda")
    calls = []
    orig_resolve = rt._resolve
    rt._resolve = lambda *a, **kw: (calls.append(1), orig_resolve(*a, **kw))[1]
    for i in range(3):
        a = eas.tensor(np.random.default_rng(i).standard_normal(hi - lo).astype(np.float32), device="cuda")
        lib.current = k.compile(a, b, c, n, BLOCK=256)
        assert run_shard(k, a, b, c, n, BLOCK=256, _rank=rank, _world=world, _buffer_base=base) == (lo // 256,
                                                                                                   hi // 256)
        np.testing.assert_array_equal(c.numpy(), a.numpy() + 1.0)
    assert len(calls) == 1
    (fl, _r), = [v for kk, v in k._fast.items() if kk[0] == "shard"]
    assert [o[3] for o in fl.ptr_slots] == [4 * lo] * 3


@eas.kernel
def add_default_block(a, b, c, N, BLOCK: eas.constexpr = 256):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


def test_run_shard_tunes_an_autotuned_kernel_on_its_own_range(fast, monkeypatch):
    """An autotuned kernel under run_shard is timed on this rank's program range (the whole launch
    may not fit the slice buffers), keeps the fastest config per range, and then launches it."""
    from easy_as_b200.shard import element_range, run_shard

    lib, rt = fast
    n, world, rank = 1 << 14, 2, 1
    tuned = eas.autotune(configs=[eas.Config(meta={"BLOCK": 256}), eas.Config(meta={"BLOCK": 512})],
                         key=["N"], warmup=1, repeat=2)(eas.kernel(add_default_block.fn))
    lo, hi = element_range(n, 512, rank, world)           # both configs split at the same element
    a = eas.tensor(np.arange(hi - lo, dtype=np.float32), device="cuda")
    b = eas.tensor(np.ones(hi - lo, np.float32), device="cuda")
    c = eas.tensor(np.zeros(hi - lo, np.float32), device="cuda")
    timed = []

    def fake_bench(ck, runtime_args, meta, *, axis, lo, hi, repeat, warmup, **kw):
        timed.append((meta["BLOCK"], axis, lo, hi))
        return 1.0 if meta["BLOCK"] == 256 else 0.5      # BLOCK 512 "wins"

    monkeypatch.setattr(rt, "benchmark_range", fake_bench)
    monkeypatch.setenv("EAS_AUTOTUNE_CACHE", "0")
    orig_raw = rt._launch_generic_raw

    def raw(ck, *a_, **kw):      # the fake decodes each launch with the kernel being launched
        lib.current = ck
        return orig_raw(ck, *a_, **kw)

    monkeypatch.setattr(rt, "_launch_generic_raw", raw)
    r = run_shard(tuned, a, b, c, n, _rank=rank, _world=world, _buffer_base={"a": lo, "b": lo, "c": lo})
    assert timed == [(256, 0, 32, 64), (512, 0, 16, 32)]     # each config's own range of rank 1
    assert r == (16, 32)
    np.testing.assert_array_equal(c.numpy(), a.numpy() + 1.0)
    (best,) = tuned._tuned_cache.values()
    assert best.meta == {"BLOCK": 512}
    (times,) = tuned._tuned_times.values()
    assert times == [({"BLOCK": 256}, 1.0), ({"BLOCK": 512}, 0.5)]



def test_unaligned_dot_gemm_operands_are_repitched_then_run_natively(fast):
    """K = 45 (A rows 90 bytes apart) and N = 300 (B rows 600 bytes apart): TMA cannot read them in
    place, so the launch re-pitches them into scratch rows padded to 8 elements and runs the native
    GEMM on the copies; the result equals the float64 product of the original operands."""
    from examples.matmul_dot_f16 import grid, matmul_dot_f16

    lib, rt = fast
    batch, M, N, K = 2, 20, 300, 45
    rng = np.random.default_rng(3)
    a = eas.tensor((rng.standard_normal(batch * M * K) / K ** 0.5).astype(np.float16), device="cuda")
    b = eas.tensor((rng.standard_normal(batch * K * N) / K ** 0.5).astype(np.float16), device="cuda")
    c = eas.tensor(np.zeros(batch * M * N, np.float32), device="cuda")
    ck = matmul_dot_f16.compile(a, b, c, M, N, K, BLOCK_N=128)
    lib.current = ck
    rt.run(ck, {"a": a, "b": b, "c": c, "M": M, "N": N, "K": K}, {"BLOCK_N": 128}, sync=True, grid=grid(batch)(
        {"BLOCK_N": 128}, {"N": N, "M": M}))
    pads = [x for x in lib.calls if x[0] == "pad_f16"]
    assert [x[1:] for x in pads] == [(M, 48, batch), (K, 304, batch)]      # A rows, then B rows
    assert [x for x in lib.calls if x[0] == "gemm"]
    want = np.matmul(a.numpy().reshape(batch, M, K).astype(np.float64), b.numpy().reshape(batch, K, N).astype(np.float64))
    np.testing.assert_allclose(c.numpy().reshape(batch, M, N), want, rtol=1e-5, atol=1e-5)
