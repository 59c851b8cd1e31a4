"""GPU: SPMD kernels with constexpr loops give the same bits re-rolled and straight-line, equal
to a sequential float32 computation."""

import numpy as np
import pytest

import spmd_loops
from easy_as_b200.compiler import compile_ir

pytestmark = pytest.mark.gpu


def _both(cuda_rt, monkeypatch, kernel, args, meta, out_name, out_size):
    ir = kernel.compile(*args.values(), **meta).ir
    outs = []
    for reroll in ("1", "0"):
        monkeypatch.setenv("EAS_REROLL", reroll)
        ck = compile_ir(ir)
        assert ("eas_r" in ck.src) == (reroll == "1")
        out = np.zeros(out_size, np.float32)
        cuda_rt.run(ck, {**args, out_name: out}, meta, sync=True)
        outs.append(out)
    return outs


@pytest.mark.parametrize("n", [1000, 4099])
def test_colsum_rerolled_equals_straight_line(cuda_rt, monkeypatch, n):
    W = 48
    rng = np.random.default_rng(n)
    x = rng.standard_normal(W * n).astype(np.float32)
    rolled, flat = _both(cuda_rt, monkeypatch, spmd_loops.colsum, {"x": x, "y": np.zeros(n, np.float32), "N": n},
                         {"W": W, "BLOCK": 256}, "y", n)
    np.testing.assert_array_equal(rolled, flat)
    want = x[:n].copy()
    for j in range(1, W):
        want = (want + x[j * n:(j + 1) * n]).astype(np.float32)
    np.testing.assert_array_equal(rolled, want)


def test_store_in_every_step(cuda_rt, monkeypatch):
    W, n = 40, 3001
    rng = np.random.default_rng(1)
    x = rng.standard_normal(W * n).astype(np.float32)
    rolled, flat = _both(cuda_rt, monkeypatch, spmd_loops.rows_scale,
                         {"x": x, "y": np.zeros(W * n, np.float32), "N": n}, {"W": W, "BLOCK": 512}, "y", W * n)
    np.testing.assert_array_equal(rolled, flat)
    np.testing.assert_array_equal(rolled, (x * np.float32(2.0) + np.float32(1.0)).astype(np.float32))
