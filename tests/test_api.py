"""Host-side API behaviour (CPU only): the behaviours the reference's own unit tests check
(tests/test_autotune.py, test_kernel_cache.py, test_grid_infer.py, test_tensor_f16.py,
test_dlpack.py, test_torch_interop.py cpu part, test_thread_id_rewrite.py), restated."""

from unittest import mock

import numpy as np
import pytest

import eas
from eas import mk
from easy_as_b200.ir import DType, IRModule, Inst, ValueRef
from easy_as_b200.runtime import get_runtime
from easy_as_b200.runtime.grid import infer_grid


class FakeRuntime:
    def __init__(self):
        self.bench, self.runs = [], []

    def benchmark(self, ck, runtime_args, meta, *, repeat, warmup=0, **kw):
        self.bench.append(dict(meta))
        return 1.0 / meta["BLOCK"]

    def run(self, ck, runtime_args, meta, **kw):
        self.runs.append(dict(meta))


def _tuned():
    @eas.autotune(configs=[eas.Config(meta={"BLOCK": b}) for b in (64, 128, 256)], key=["N"], warmup=0, repeat=1)
    @eas.kernel
    def addk(a, b, c, N, BLOCK: eas.constexpr = 64):
        offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
        m = offs < N
        mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)

    return addk


def test_autotune_selects_and_caches_per_key(monkeypatch):
    monkeypatch.setenv("EAS_AUTOTUNE_CACHE", "0")
    k = _tuned()
    rt = FakeRuntime()
    with mock.patch("eas.kernel.get_runtime", return_value=rt):
        a = np.zeros(1027, np.float32)
        k(a, a, a, 1027)
        assert len(rt.bench) == 3 and rt.runs[-1]["BLOCK"] == 256
        k(a, a, a, 1027)
        assert len(rt.bench) == 3
        b = np.zeros(2055, np.float32)
        k(b, b, b, 2055)
        assert len(rt.bench) == 6 and rt.runs[-1]["BLOCK"] == 256


def test_autotune_disk_cache(monkeypatch, tmp_path):
    monkeypatch.setenv("EAS_CACHE_DIR", str(tmp_path))
    monkeypatch.delenv("EAS_AUTOTUNE_CACHE", raising=False)
    a = np.zeros(100, np.float32)
    rt = FakeRuntime()
    with mock.patch("eas.kernel.get_runtime", return_value=rt):
        _tuned()(a, a, a, 100)
        assert len(rt.bench) == 3
        _tuned()(a, a, a, 100)  # a new Kernel object: result comes from disk
        assert len(rt.bench) == 3 and rt.runs[-1]["BLOCK"] == 256
    assert (tmp_path / "autotune.json").exists()


def test_autotune_argument_checks():
    with pytest.raises(ValueError):
        eas.autotune(configs=[], key=["N"])
    with pytest.raises(ValueError):
        eas.autotune(configs=[eas.Config(meta={})], key=[])


@eas.kernel
def axpy(a, b, c, N, alpha, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) * alpha + mk.load(b, offs, m), m)


def test_compile_cache_ignores_scalar_values():
    a = np.zeros(10, np.float32)
    assert axpy.compile(a, a, a, 10, 2.0, BLOCK=256) is axpy.compile(a, a, a, 10, 3.0, BLOCK=256)
    assert axpy.compile(a, a, a, 10, 2.0, BLOCK=256) is not axpy.compile(a, a, a, 10, 2.0, BLOCK=128)


@eas.kernel
def add2d(a, b, c, H, W, BLOCK: eas.constexpr):
    col = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    row = mk.program_id(1)
    offs = row * W + col
    m = mk.where(row < H, col < W, False)
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


def test_grid_inference():
    a = np.zeros(17 * 103, np.float32)
    ck = add2d.compile(a, a, a, 17, 103, BLOCK=32)
    assert infer_grid(ck.ir, {"H": 17, "W": 103}, ck.block_size) == (4, 17, 1)
    assert infer_grid(ck.ir, {}, 16, shape=(9, 65)) == (5, 9, 1)
    with pytest.raises(ValueError):
        infer_grid(ck.ir, {}, 16)


def test_launch_option_validation():
    a = np.zeros(8, np.float32)
    with pytest.raises(ValueError):
        add2d(a, a, a, 2, 4, BLOCK=4, _tptg=(8, 1, 1))
    with pytest.raises(TypeError):
        add2d(a, a, a, 2, 4, BLOCK=4, _sync="yes")
    with pytest.raises(ValueError):
        add2d(a, a, a, 2, 4, BLOCK=4, _grid=(1, 2, 3, 4))


def test_thread_id_rewrite_needs_one_tid_size():
    from eas.compiler import _rewrite_thread_id

    pid, blk, mul, t0, t1, out = (ValueRef(i, DType.U32) for i in range(1, 7))
    multi = IRModule("k", (), (Inst("program_id", pid, (0,)), Inst("const", blk, (256,)), Inst("mul", mul, (pid, blk)),
                               Inst("tid", t0, (0, 256)), Inst("tid", t1, (0, 128)), Inst("add", out, (mul, t0))))
    assert _rewrite_thread_id(multi).insts[-1].op == "add"
    single = IRModule("k", (), tuple(i for i in multi.insts if i.out is not t1))
    assert _rewrite_thread_id(single).insts[-1].op == "thread_id"


def test_thread_id_rewrite_env_disable(monkeypatch):
    monkeypatch.setenv("EAS_DISABLE_THREAD_ID_REWRITE", "1")

    @eas.kernel
    def k(a, b, c, N, BLOCK: eas.constexpr):
        offs = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
        m = offs < N
        mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)

    a = np.zeros(4, np.float32)
    assert "thread_id" not in [i.op for i in k.compile(a, a, a, 4, BLOCK=256).ir.insts]


def test_cpu_tensors_and_dlpack():
    a = np.random.default_rng(0).standard_normal(1024).astype(np.float32)
    t = eas.tensor(a, device="cpu")
    assert type(eas.to_dlpack(t)).__name__ == "PyCapsule"
    np.testing.assert_array_equal(np.from_dlpack(t), a)
    np.testing.assert_array_equal(eas.from_dlpack(a).numpy(), a)
    h = np.random.default_rng(1).standard_normal(128).astype(np.float16)
    th = eas.tensor(h, device="cpu")
    assert th.dtype == np.float16 and np.from_dlpack(th).dtype == np.float16
    e = eas.empty((16, 8), device="cpu", dtype=np.float16)
    assert e.numpy().dtype == np.float16 and e.shape == (16, 8)
    with pytest.raises(TypeError):
        eas.tensor(np.zeros(3, np.float64), dtype=np.float64)


def test_torch_cpu_zero_copy_wrap():
    import torch

    t = torch.zeros(1027)
    e = eas.tensor(t, device="cpu")
    t.add_(1.0)
    np.testing.assert_array_equal(e.numpy(), t.numpy())
    e.numpy()[0] = 7.0
    assert float(t[0]) == 7.0


def test_backend_selection_errors():
    with pytest.raises(ValueError, match="cpu"):
        get_runtime("cpu")
    with pytest.raises(ValueError):
        get_runtime("mps")
    with pytest.raises(ValueError):
        get_runtime("vulkan")


def test_mk_outside_trace_raises():
    with pytest.raises(RuntimeError):
        mk.program_id(0)


def test_unsupported_buffer_dtype():
    @eas.kernel
    def k(x, N, BLOCK: eas.constexpr):
        mk.store(x, mk.tid(0, BLOCK), 1.0, True)

    with pytest.raises(TypeError):
        k.compile(np.zeros(4, np.float64), 4, BLOCK=32)


@eas.kernel
def _in_tile_store_kernel(src, dst, LIMIT: eas.constexpr, NT: eas.constexpr):
    tid = mk.tid(0, NT)
    for i in range(0, LIMIT, NT):
        idx = tid + i
        in_tile = idx < LIMIT
        mk.store(dst, idx, mk.load(src, idx, True), in_tile)


@pytest.mark.parametrize("limit,folded", [(64, True), (70, False)])
def test_interval_lt_fold(limit, folded):
    """A `tid + i < LIMIT` bound that holds for every thread (LIMIT a multiple of NT) is folded
    away; otherwise it stays (reference tests/test_interval_lt_fold.py:23-36)."""
    src = np.arange(limit, dtype=np.float32)
    ck = _in_tile_store_kernel.compile(src, np.zeros_like(src), LIMIT=limit, NT=16)
    assert ("lt" in [i.op for i in ck.ir.insts]) is not folded


def test_launch_path_environment_lookups_follow_os_environ(monkeypatch):
    """The launch path reads EAS_* switches through runtime.env_bytes, which must see every change
    made through os.environ (as monkeypatch, or a user, makes them)."""
    from easy_as_b200.runtime import env_bytes

    monkeypatch.delenv("EAS_BOUNDS_CHECK", raising=False)
    assert env_bytes(b"EAS_BOUNDS_CHECK") is None
    monkeypatch.setenv("EAS_BOUNDS_CHECK", "1")
    assert env_bytes(b"EAS_BOUNDS_CHECK") == b"1"
    monkeypatch.setenv("EAS_BOUNDS_CHECK", "0")
    assert env_bytes(b"EAS_BOUNDS_CHECK") == b"0"
