"""GPU: the reference's masked tiled, naive and dot matmul kernels (IR from the reference front
end) on the proven-GEMM FFMA path give the same bits as their generated kernels, and as the CPU
oracle at the golden sizes."""

from __future__ import annotations

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from oracle.interp import execute

pytestmark = pytest.mark.gpu


def _cdiv(a, b):
    return -(-a // b)


# case id, scalar values, grid (None: inferred), buffer sizes
CASES = [
    ("matmul_tiled_masked", {"M": 50, "N": 72, "PID_M_BASE": 0, "PID_N_BASE": 0}, (_cdiv(72, 64), _cdiv(50, 16), 1),
     {"a": 50 * 64, "b": 64 * 72, "c": 50 * 72}),
    ("matmul_tiled_masked", {"M": 300, "N": 260, "PID_M_BASE": 0, "PID_N_BASE": 0},
     (_cdiv(260, 64), _cdiv(300, 16), 1), {"a": 300 * 64, "b": 64 * 260, "c": 300 * 260}),
    ("matmul_tiled_masked", {"M": 300, "N": 260, "PID_M_BASE": 2, "PID_N_BASE": 1}, (2, 5, 1),
     {"a": 300 * 64, "b": 64 * 260, "c": 300 * 260}),
    ("matmul_naive", {"H": 40, "W": 72}, None, {"a": 40 * 16, "b": 16 * 72, "c": 40 * 72}),
    # rows not 16-byte aligned: element-wise staging
    ("matmul_tiled_masked", {"M": 50, "N": 70, "PID_M_BASE": 0, "PID_N_BASE": 0}, (_cdiv(70, 64), _cdiv(50, 16), 1),
     {"a": 50 * 64, "b": 64 * 70, "c": 50 * 70}),
    ("t_matmul_tiled", {"M": 17, "N": 130}, (_cdiv(130, 64), _cdiv(17, 16), 1), {"a": 17 * 31, "b": 31 * 130,
                                                                                "c": 17 * 130}),
    ("t_matmul_tiled_33x65x48", {"M": 33, "N": 65}, (_cdiv(65, 64), _cdiv(33, 16), 1),
     {"a": 33 * 48, "b": 48 * 65, "c": 33 * 65}),
    ("matmul_naive", {"H": 40, "W": 70}, None, {"a": 40 * 16, "b": 16 * 70, "c": 40 * 70}),
    ("t_matmul", {"M": 32, "N": 100}, (32, 2, 1), {"a": 32 * 16, "b": 16 * 100, "c": 32 * 100}),
    ("t_fma_matmul", {"M": 32, "N": 64}, (32, 2, 1), {"a": 32 * 8, "b": 8 * 64, "c": 32 * 64}),
]


@pytest.mark.parametrize("cid,scal,grid,sizes", CASES, ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_native_matches_generated_kernel(cuda_rt, monkeypatch, cid, scal, grid, sizes):
    import torch

    c = goldens.case(cid)
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    assert ck.plan.native is not None and ck.plan.native.kind == "tiled_f32_ffma"
    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(sizes["a"], device="cuda", generator=g)
    b = torch.randn(sizes["b"], device="cuda", generator=g)
    opts = {} if grid is None else {"grid": grid}
    outs = []
    for disable in ("0", "1"):
        monkeypatch.setenv("EAS_DISABLE_NATIVE", disable)
        out = torch.full((sizes["c"],), float("nan"), device="cuda")
        before = cuda_rt.native_launches
        cuda_rt.run(ck, {"a": a, "b": b, "c": out, **scal}, c["meta"], sync=True, **opts)
        took_native = cuda_rt.native_launches == before + 1
        assert took_native == (disable == "0"), ck.plan.native.last_reason
        outs.append(out)
    # compare bit patterns: the NaN fill stays where neither kernel stores
    assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32))


@pytest.mark.parametrize("cid", ["matmul_tiled_full", "t_fma_matmul", "t_matmul"])
def test_golden_size_native_launch_matches_oracle(cuda_rt, cid):
    c = goldens.case(cid)
    ir = goldens.ir_from_json(c["opt"])
    ck = compile_ir(ir)
    inp = goldens.make_inputs(c, 4)
    cpu = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in inp.items()}
    before = cuda_rt.native_launches
    cuda_rt.run(ck, inp, c["meta"], sync=True, **goldens.launch_opts(c))
    assert cuda_rt.native_launches == before + 1, ck.plan.native.last_reason
    execute(ir, cpu, **goldens.launch_opts(c))
    for name in c["writes"]:
        np.testing.assert_array_equal(inp[name], cpu[name])
