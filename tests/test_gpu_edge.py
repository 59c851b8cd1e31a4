"""GPU edge cases, each checked bit for bit against the CPU oracle: empty launches, ragged
and non-multiple-of-4 BLOCKs, f16 data, scalar kinds, u32 corner semantics, grids taller than
65535, partial thread groups with barriers."""

import numpy as np
import pytest

import eas
from eas import mk
from oracle.interp import execute

pytestmark = pytest.mark.gpu


def _both(kernel, args, meta, **launch):
    """Run on the GPU (numpy buffers) and in the oracle; return (gpu_args, oracle_args)."""
    g = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in args.items()}
    o = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in args.items()}
    kernel(**g, **meta, **{f"_{k}": v for k, v in launch.items()})
    ck = kernel.compile(**o, **meta)
    execute(ck.ir, o, **launch)
    return g, o


@eas.kernel
def axpb(x, y, N, alpha, beta, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(y, offs, mk.fma(mk.load(x, offs, m), alpha, beta), m)


@pytest.mark.parametrize("block", [1, 12, 250, 1000, 2000, 4096])
@pytest.mark.parametrize("n", [0, 1, 5, 4099])
def test_spmd_ragged_blocks(cuda_rt, block, n):
    rng = np.random.default_rng(block + n)
    args = {"x": rng.standard_normal(max(n, 1), dtype=np.float32), "y": np.zeros(max(n, 1), np.float32), "N": n,
            "alpha": 1.25, "beta": -0.5}
    g, o = _both(axpb, args, {"BLOCK": block})
    np.testing.assert_array_equal(g["y"], o["y"])


@eas.kernel
def add_f16(a, b, c, N, BLOCK: eas.constexpr):
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < N
    mk.store(c, offs, mk.load(a, offs, m) + mk.load(b, offs, m), m)


def test_f16_vector_path(cuda_rt):
    rng = np.random.default_rng(3)
    n = 10_007
    args = {"a": rng.standard_normal(n).astype(np.float16), "b": rng.standard_normal(n).astype(np.float16),
            "c": np.zeros(n, np.float16), "N": n}
    g, o = _both(add_f16, args, {"BLOCK": 512})
    np.testing.assert_array_equal(g["c"], o["c"])
    np.testing.assert_array_equal(g["c"], (args["a"].astype(np.float32) + args["b"].astype(np.float32)).astype(np.float16))


@eas.kernel
def u32_corners(x, out, N, d, BLOCK: eas.constexpr):
    i = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    m = i < N
    v = mk.to_u32(mk.load(x, i, m))  # truncating, saturating float -> u32
    q = v // d
    r = v % d
    mk.store(out, i * 3, mk.to_f32(v), m)
    mk.store(out, i * 3 + 1, mk.to_f32(q), m)
    mk.store(out, i * 3 + 2, mk.to_f32(r), m)


@pytest.mark.parametrize("d", [0, 1, 7])
def test_u32_casts_and_division(cuda_rt, d):
    x = np.array([-3.7, -0.0, 0.9, 1.5, 123456.7, 4.3e9, 5e9, np.nan, np.inf, -np.inf, 65535.5], np.float32)
    args = {"x": x, "out": np.zeros(3 * x.size, np.float32), "N": x.size, "d": d}
    g, o = _both(u32_corners, args, {"BLOCK": 64})
    np.testing.assert_array_equal(g["out"], o["out"])


@eas.kernel
def scalar_kinds(out, N, h, flag, BLOCK: eas.constexpr):
    i = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    hv = mk.to_f32(h) + mk.to_f32(flag)
    mk.store(out, i, hv * mk.to_f32(i), i < N)


def test_f16_and_bool_scalars(cuda_rt):
    args = {"out": np.zeros(100, np.float32), "N": 100, "h": np.float16(1.5), "flag": True}
    g, o = _both(scalar_kinds, args, {"BLOCK": 32})
    np.testing.assert_array_equal(g["out"], o["out"])


@eas.kernel
def tall_grid(out, H, W, BLOCK: eas.constexpr):
    col = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    row = mk.program_id(1)
    mk.store(out, row * W + col, mk.to_f32(row), (row < H) & (col < W))


def test_grid_taller_than_65535(cuda_rt):
    H, W = 70_001, 3
    out = np.full(H * W, -1, np.float32)
    tall_grid(out, H, W, BLOCK=32)
    np.testing.assert_array_equal(out, np.repeat(np.arange(H, dtype=np.float32), W))


@eas.kernel
def rev_in_block(x, y, N, BLOCK: eas.constexpr):
    t = mk.tid(0, BLOCK)
    i = mk.program_id(0) * BLOCK + t
    s = mk.alloc_tg(BLOCK)
    mk.store(s, t, mk.load(x, i, i < N))
    mk.barrier()
    # swap neighbours inside the group: thread t reads the slot thread t^1 wrote
    j = t + 1 + (t % 2) * 0xFFFFFFFE  # t + 1 - 2 * (t % 2), with u32 wraparound
    mk.store(y, i, mk.load(s, j), i < N)


@pytest.mark.parametrize("n", [64, 100, 1000])  # even n: every partner thread exists
def test_partial_group_with_barrier(cuda_rt, n):
    rng = np.random.default_rng(n)
    args = {"x": rng.standard_normal(n, dtype=np.float32), "y": np.zeros(n, np.float32), "N": n}
    g, o = _both(rev_in_block, args, {"BLOCK": 64})
    np.testing.assert_array_equal(g["y"], o["y"])


def test_zero_size_grid_is_a_no_op(cuda_rt):
    out = np.full(4, 7, np.float32)
    tall_grid(out, 0, 4, BLOCK=32)
    tall_grid(out, 4, 4, BLOCK=32, _grid=(0, 4, 1))
    np.testing.assert_array_equal(out, np.full(4, 7, np.float32))
