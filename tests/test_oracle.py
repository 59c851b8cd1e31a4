"""Pin the CPU oracle (oracle/interp.py) before trusting it.

Each case executes the reference front end's own IR (golden fixtures) in the
oracle and checks the known answers the reference's tests assert:
exact a+b (tests/test_add.py:38 uses assert_allclose with rtol 1e-7; here it is
bit-exact), arange % BLOCK (test_local_and_lane_id.py:53), arange % 32
(:73), identity copy (test_threadgroup_memory.py:89), row-index fill
(test_callable_grid.py:51-52), arange(n) (test_tptg_override.py:47-49),
GEMV (test_dot_dynamic_k.py:45, rtol 1e-4), matmuls vs float64
(test_matmul.py:55-56 rtol 1e-4/atol 1e-5; test_matmul_tiled.py:173 2e-3;
examples/matmul_simdgroup.py:224 5e-3 vs f16-cast inputs).
"""

from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest

import goldens
from oracle.interp import execute, fma_f32


def run(cid, seed=0):
    c = goldens.case(cid)
    inp = goldens.make_inputs(c, seed)
    execute(goldens.ir_from_json(c["opt"]), inp, **goldens.launch_opts(c))
    return c, inp


@pytest.mark.parametrize("cid", ["add_c1", "add_block1024", "t_add"])
def test_add_exact(cid):
    _, x = run(cid)
    np.testing.assert_array_equal(x["c"], x["a"] + x["b"])


def test_add_c1_is_config1():
    c = goldens.case("add_c1")
    assert c["args"][3] == 1031 and c["meta"]["BLOCK"] == 256


def test_local_and_lane_ids():
    _, x = run("t_local_id")
    np.testing.assert_array_equal(x["out"], (np.arange(384) % 128).astype(np.float32))
    _, x = run("t_lane_id")
    np.testing.assert_array_equal(x["out"], (np.arange(256) % 32).astype(np.float32))


@pytest.mark.parametrize("cid", ["t_tg_copy", "t_tg_copy_masked"])
def test_tg_copy(cid):
    _, x = run(cid)
    np.testing.assert_array_equal(x["out"], x["a"])


def test_callable_grid_rows():
    _, x = run("t_callable_grid")
    np.testing.assert_array_equal(x["out"].reshape(5, 10), np.repeat(np.arange(5, dtype=np.float32), 10).reshape(5, 10))


def test_tptg_arange():
    _, x = run("t_tptg")
    np.testing.assert_array_equal(x["out"], np.arange(1031, dtype=np.float32))


def test_gemv():
    _, x = run("t_gemv_dot")
    a = x["a"].reshape(33, 31).astype(np.float64)
    np.testing.assert_allclose(x["y"], a @ x["x"].astype(np.float64), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("cid,m,n,k,tol", [("matmul_naive", 40, 70, 16, 1e-4), ("t_matmul", 32, 100, 16, 1e-4),
                                           ("t_fma_matmul", 32, 64, 8, 1e-4),
                                           ("matmul_tiled_masked", 50, 70, 64, 2e-3),
                                           ("matmul_tiled_full", 64, 128, 64, 2e-3),
                                           ("t_matmul_tiled", 17, 130, 31, 2e-3)])
def test_matmuls(cid, m, n, k, tol):
    _, x = run(cid)
    ref = x["a"].reshape(m, k).astype(np.float64) @ x["b"].reshape(k, n).astype(np.float64)
    np.testing.assert_allclose(x["c"].reshape(m, n), ref, rtol=tol, atol=tol)


def test_simdgroup_matmul():
    _, x = run("matmul_simdgroup")
    a = x["a"].reshape(40, 32).astype(np.float16).astype(np.float64)
    b = x["b"].reshape(32, 36).astype(np.float16).astype(np.float64)
    np.testing.assert_allclose(x["c"].reshape(40, 36), a @ b, rtol=5e-3, atol=5e-3)


def test_fma_kernels():
    _, x = run("t_fma_simple")
    np.testing.assert_array_equal(x["d"], fma_f32(x["a"], x["b"], x["c"]))
    np.testing.assert_allclose(x["d"], x["a"] * x["b"] + x["c"], rtol=1e-5, atol=1e-6)


def test_axpy_scalar_arg():
    _, x = run("t_axpy")
    np.testing.assert_array_equal(x["c"], fma_f32(x["a"], np.float32(2.0), x["b"]))


def test_in_tile_kernels():
    _, x = run("t_in_tile_fold")
    np.testing.assert_array_equal(x["dst"], x["src"])
    _, x = run("t_in_tile_keep")
    np.testing.assert_array_equal(x["dst"][:70], x["src"][:70])
    assert not x["dst"][70:].any()


def test_bool_kernels():
    _, x = run("t_bool_simplify")
    np.testing.assert_array_equal(x["out"], (np.arange(256) < 128).astype(np.float32))
    _, x = run("t_bool_chain")
    np.testing.assert_array_equal(x["out"], (np.arange(256) < 128).astype(np.float32))


def test_many_dot_zero_smem():
    _, x = run("t_many_dot")
    assert x["out"][0] == 0.0


def _exact_fma(a, b, c):
    v = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    # round the exact rational to float32 (nearest, ties to even) by bracketing
    f = np.float32(float(v))
    lo = np.nextafter(f, np.float32(-np.inf))
    hi = np.nextafter(f, np.float32(np.inf))
    best = min((f, lo, hi), key=lambda y: (abs(Fraction(float(y)) - v), int(np.array(y).view(np.uint32)) & 1))
    return best


def test_fma_f32_is_correctly_rounded():
    rng = np.random.default_rng(7)
    a = rng.standard_normal(3000).astype(np.float32)
    b = rng.standard_normal(3000).astype(np.float32)
    c = (rng.standard_normal(3000) * 10.0 ** rng.integers(-8, 8, 3000)).astype(np.float32)
    got = fma_f32(a, b, c)
    for i in range(3000):
        assert got[i] == _exact_fma(a[i], b[i], c[i]), i


def test_fma_f32_midpoint_cases():
    # p + c lands on a float32 midpoint in float64 while the exact value does not
    a = np.float32(1 + 2 ** -12)
    b = np.float32(1 + 2 ** -12)
    for c in (np.float32(2 ** -24), np.float32(-(2 ** -24)), np.float32(2 ** -48), np.float32(3 * 2 ** -25)):
        assert fma_f32(a, b, c) == _exact_fma(a, b, c)
