"""GPU parity: the reference's own kernels (as IR from its front end) run through the
CUDA emitter + runtime on the B200 and match the CPU oracle on identical seeded inputs.

Bit-exact for everything except the simdgroup-MMA kernel, whose reference
summation order is unspecified (tolerance 5e-3 vs the oracle, as
examples/matmul_simdgroup.py:224 uses against an f16-cast reference).
"""

from __future__ import annotations

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from oracle.interp import execute

pytestmark = pytest.mark.gpu
CASES = goldens.cases()
TOLERANT = {"matmul_simdgroup": 5e-3}
# kernels whose output is undefined in the reference too: t_many_dot sums dots over
# threadgroup memory it never writes (reference tests/test_dot_codegen_unique_vars.py only
# inspects its generated source), so only compile + launch is checked
UNDEFINED = {"t_many_dot"}


def _run_both(rt, c, seed, to_torch=False):
    ir = goldens.ir_from_json(c["opt"])
    ck = compile_ir(ir)
    gpu_in = goldens.make_inputs(c, seed)
    cpu_in = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in gpu_in.items()}
    opts = goldens.launch_opts(c)
    if to_torch:
        import torch

        tin = {k: (torch.from_numpy(v).cuda() if isinstance(v, np.ndarray) else v) for k, v in gpu_in.items()}
        rt.run(ck, tin, c["meta"], sync=True, **opts)
        gpu_in = {k: (v.cpu().numpy() if hasattr(v, "cpu") else v) for k, v in tin.items()}
    else:
        rt.run(ck, gpu_in, c["meta"], sync=True, **opts)
    execute(ir, cpu_in, **opts)
    return gpu_in, cpu_in


@pytest.mark.parametrize("c", CASES, ids=[c["id"] for c in CASES])
def test_reference_kernel_matches_oracle(cuda_rt, c):
    for seed in (0, 1):
        gpu, cpu = _run_both(cuda_rt, c, seed)
        for name in c["writes"]:
            if c["id"] in UNDEFINED:
                continue
            if c["id"] in TOLERANT:
                np.testing.assert_allclose(gpu[name], cpu[name], rtol=TOLERANT[c["id"]], atol=TOLERANT[c["id"]])
            else:
                np.testing.assert_array_equal(gpu[name], cpu[name], err_msg=f"{c['id']}:{name}")


@pytest.mark.parametrize("cid", ["add_c1", "t_tg_copy", "matmul_tiled_masked", "matmul_simdgroup", "t_gemv_dot"])
def test_torch_cuda_tensors_zero_copy(cuda_rt, cid):
    c = goldens.case(cid)
    gpu, cpu = _run_both(cuda_rt, c, 3, to_torch=True)
    for name in c["writes"]:
        tol = TOLERANT.get(cid, 0)
        np.testing.assert_allclose(gpu[name], cpu[name], rtol=tol, atol=tol)


def test_add_config1_known_answer(cuda_rt):
    """N=1031, BLOCK=256, a,b ~ N(0,1) from seed 0; bit-exact c = a + b."""
    c = goldens.case("add_c1")
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    rng = np.random.default_rng(0)
    a = rng.standard_normal(1031, dtype=np.float32)
    b = rng.standard_normal(1031, dtype=np.float32)
    out = np.zeros_like(a)
    cuda_rt.run(ck, {"a": a, "b": b, "c": out, "N": 1031}, {"BLOCK": 256})
    np.testing.assert_array_equal(out, a + b)


@pytest.mark.parametrize("cid", ["matmul_naive", "matmul_tiled_masked", "t_fma_matmul", "t_matmul"])
def test_rerolled_and_unrolled_sources_agree(cuda_rt, cid, monkeypatch):
    """Kernels whose unrolled constexpr loops the emitter prints as loops give the same bits
    as the straight-line source (EAS_REROLL=0)."""
    c = goldens.case(cid)
    ir = goldens.ir_from_json(c["opt"])
    rolled = compile_ir(ir)
    monkeypatch.setenv("EAS_REROLL", "0")
    flat = compile_ir(ir)
    assert "eas_r" in rolled.src and "eas_r" not in flat.src
    outs = []
    for ck in (rolled, flat):
        inp = goldens.make_inputs(c, 5)
        cuda_rt.run(ck, inp, c["meta"], sync=True, **goldens.launch_opts(c))
        outs.append(inp)
    for name in c["writes"]:
        np.testing.assert_array_equal(outs[0][name], outs[1][name])


@pytest.mark.parametrize("cid", ["t_matmul_tiled_33x65x48", "t_matmul_tiled_64x64x32", "t_matmul_tiled"])
def test_reference_tiled_matmul_device_check(cuda_rt, cid):
    """The reference test's own device check (tests/test_matmul_tiled.py:128-178): shapes
    (33,65,48), (64,64,32), (17,130,31), BM=16 BN=64 BK=16 NT=256, against a @ b with rtol=atol=2e-3;
    here also bit for bit against the oracle."""
    c = goldens.case(cid)
    ir = goldens.ir_from_json(c["opt"])
    M, N = c["args"][3], c["args"][4]
    K = c["meta"]["K"]
    rng = np.random.default_rng(5)
    a = rng.standard_normal(M * K).astype(np.float32)
    b = rng.standard_normal(K * N).astype(np.float32)
    gpu = np.zeros(M * N, np.float32)
    cpu = np.zeros(M * N, np.float32)
    cuda_rt.run(compile_ir(ir), {"a": a, "b": b, "c": gpu, "M": M, "N": N}, c["meta"], sync=True,
                **goldens.launch_opts(c))
    execute(ir, {"a": a, "b": b, "c": cpu, "M": M, "N": N}, **goldens.launch_opts(c))
    np.testing.assert_array_equal(gpu, cpu)
    want = a.reshape(M, K).astype(np.float64) @ b.reshape(K, N).astype(np.float64)
    np.testing.assert_allclose(gpu.reshape(M, N), want, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("k", [7, 31, 64])
def test_reference_dot_dynamic_k_device_check(cuda_rt, k):
    """tests/test_dot_dynamic_k.py:27-50: gemv with a runtime K in {7, 31, 64}, M = 33, BLOCK = 64,
    rtol=atol=1e-4 against a @ x; here also bit for bit against the oracle."""
    c = goldens.case("t_gemv_dot")
    ir = goldens.ir_from_json(c["opt"])
    m = 33
    rng = np.random.default_rng(k)
    a = rng.standard_normal(m * k).astype(np.float32)
    x = rng.standard_normal(k).astype(np.float32)
    gpu = np.zeros(m, np.float32)
    cpu = np.zeros(m, np.float32)
    args = {"a": a, "x": x, "M": m, "K": k, "N": m}
    cuda_rt.run(compile_ir(ir), {**args, "y": gpu}, {"BLOCK": 64}, sync=True, nthreads=m)
    execute(ir, {**args, "y": cpu}, nthreads=m)
    np.testing.assert_array_equal(gpu, cpu)
    np.testing.assert_allclose(gpu, a.reshape(m, k).astype(np.float64) @ x.astype(np.float64), rtol=1e-4, atol=1e-4)
