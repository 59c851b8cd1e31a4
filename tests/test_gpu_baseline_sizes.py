"""Parity at the BASELINE configurations' full sizes, through size-independent properties.

C2: N = 2^28 f32 add, bit-exact against c = a + b.
C3: the reference's unmodified tiled fp32 kernel (IR from the reference front end, K = 2048
    constexpr, 32x32x32 tiles, NT = 256): bit-exact against the CPU oracle on a one-tile launch
    of the same IR, and the full 2048^3 product within rtol 1e-4 of float64 (north_star bar).
C4/C5: the fp16 mk.dot GEMM at 8192^3 and 64 x 4096 x 4096 x 2088, sampled rows against
    float64 (rtol 2e-2 is the north_star bar; the tensor-core result holds 1e-5 * sqrt(K/2048) normwise).
"""

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from examples.matmul_dot_f16 import grid, matmul_dot_f16
from oracle.interp import execute

pytestmark = pytest.mark.gpu


def test_c2_add_full_size(cuda_rt):
    import torch

    c = goldens.case("add_block1024")
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    n = 1 << 28
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randn(n, device="cuda", generator=g)
    b = torch.randn(n, device="cuda", generator=g)
    out = torch.empty_like(a)
    cuda_rt.run(ck, {"a": a, "b": b, "c": out, "N": n}, {"BLOCK": 1024})
    assert torch.equal(out, a + b)


def test_c3_tiled_fp32_one_tile_bit_exact(cuda_rt):
    c = goldens.case("matmul_tiled_c3_full")
    ir = goldens.ir_from_json(c["opt"])
    ck = compile_ir(ir)
    M = N = 32
    K = 2048
    rng = np.random.default_rng(2)
    a = rng.uniform(-1, 1, M * K).astype(np.float32)
    b = rng.uniform(-1, 1, K * N).astype(np.float32)
    gpu = np.zeros(M * N, np.float32)
    cpu = np.zeros(M * N, np.float32)
    cuda_rt.run(ck, {"a": a, "b": b, "c": gpu, "M": M, "N": N}, c["meta"], grid=(1, 1, 1))
    execute(ir, {"a": a, "b": b, "c": cpu, "M": M, "N": N}, grid=(1, 1, 1))
    np.testing.assert_array_equal(gpu, cpu)


def test_c3_tiled_fp32_full_size(cuda_rt):
    import torch

    c = goldens.case("matmul_tiled_c3_full")
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    M = N = K = 2048
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.rand(M * K, device="cuda", generator=g) * 2 - 1
    b = torch.rand(K * N, device="cuda", generator=g) * 2 - 1
    out = torch.zeros(M * N, device="cuda")
    cuda_rt.run(ck, {"a": a, "b": b, "c": out, "M": M, "N": N}, c["meta"], grid=(64, 64, 1))
    ref = a.double().reshape(M, K) @ b.double().reshape(K, N)
    torch.testing.assert_close(out.double().reshape(M, N), ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("batch,M,N,K", [(1, 8192, 8192, 8192), (64, 4096, 4096, 2088)])
def test_fp16_gemm_full_size_every_output_vs_float64(cuda_rt, batch, M, N, K):
    """Configs C4 and C5 at full size: EVERY output of the library's launch against a float64
    product computed on the GPU (cuBLAS DGEMM, batch by batch), at the north-star bound
    (rtol 2e-2) and at the normwise f32-accumulation bound the sampled check uses."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(5)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.empty(batch, M, N, device="cuda")
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, _grid=grid(batch))
    assert cuda_rt.native_launches == before + 1
    worst = 0.0
    for bi in range(batch):
        ref = a[bi].double() @ b[bi].double()
        got = c[bi].double()
        scale = ref.abs().max().item()
        err = (got - ref).abs()
        assert bool((err <= 2e-2 * ref.abs() + 2e-2 * scale).all()), f"batch {bi}"
        worst = max(worst, err.max().item() / scale)
        del ref, got, err
    assert worst <= 1e-5 * max(1.0, (K / 2048) ** 0.5), worst


@pytest.mark.parametrize("batch,M,N,K", [(1, 8192, 8192, 8192), (64, 4096, 4096, 2088)])
def test_fp16_gemm_full_size_sampled(cuda_rt, batch, M, N, K):
    import torch

    g = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).half()
    b = (torch.randn(batch, K, N, device="cuda", generator=g) / K ** 0.5).half()
    c = torch.empty(batch, M, N, device="cuda")
    before = cuda_rt.native_launches
    matmul_dot_f16(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, _grid=grid(batch))
    assert cuda_rt.native_launches == before + 1
    rows = torch.tensor([0, 1, M // 2, M - 1], device="cuda")
    for bi in sorted({0, batch // 2, batch - 1}):
        ref = a[bi, rows].double() @ b[bi].double()
        got = c[bi, rows].double()
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item())
        # f32 accumulation error grows like sqrt(K): 1e-5 normwise at K = 2048
        assert ((got - ref).abs().max() / ref.abs().max()).item() <= 1e-5 * max(1.0, (K / 2048) ** 0.5)


def test_c3_rerolled_loop_matches_unrolled_source_full_size(cuda_rt, monkeypatch):
    """The 2048^3 tiled kernel printed as a 63-iteration loop gives the same bits as the
    3,000-instruction straight-line source."""
    import torch

    c = goldens.case("matmul_tiled_c3_full")
    ir = goldens.ir_from_json(c["opt"])
    monkeypatch.setenv("EAS_DISABLE_NATIVE", "1")  # compare the two generic sources
    rolled = compile_ir(ir)
    monkeypatch.setenv("EAS_REROLL", "0")
    flat = compile_ir(ir)
    assert "eas_r" in rolled.src and "eas_r" not in flat.src
    M = N = K = 2048
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.rand(M * K, device="cuda", generator=g) * 2 - 1
    b = torch.rand(K * N, device="cuda", generator=g) * 2 - 1
    outs = []
    for ck in (rolled, flat):
        out = torch.zeros(M * N, device="cuda")
        cuda_rt.run(ck, {"a": a, "b": b, "c": out, "M": M, "N": N}, c["meta"], grid=(64, 64, 1))
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("mn,grid", [((2048, 2048), (64, 64, 1)), ((96, 160), (5, 3, 1)), ((32, 32), (1, 1, 1)),
                                     ((3200, 3232), (101, 100, 1))])
def test_c3_native_ffma_kernel_matches_generic_kernel_bit_for_bit(cuda_rt, monkeypatch, mn, grid):
    """The proven tiled-GEMM launch (eas_sgemm_f32_tiled) against the generated kernel of the same
    IR: identical bits, at the full 2048^3 size (64 x 64 native tiles) and at sizes that are not
    multiples of the native tile, for both tile shapes (3200 x 3232 takes the 128 x 128 tiles)."""
    import torch

    c = goldens.case("matmul_tiled_c3_full")
    ir = goldens.ir_from_json(c["opt"])
    M, N = mn
    K = 2048
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(M * K, device="cuda", generator=g)
    b = torch.randn(K * N, device="cuda", generator=g)
    ck = compile_ir(ir)
    assert ck.plan.native is not None and ck.plan.native.kind == "tiled_f32_ffma"
    before = cuda_rt.native_launches
    native = torch.full((M * N,), float("nan"), device="cuda")
    cuda_rt.run(ck, {"a": a, "b": b, "c": native, "M": M, "N": N}, c["meta"], grid=grid)
    assert cuda_rt.native_launches == before + 1, ck.plan.native.last_reason
    monkeypatch.setenv("EAS_DISABLE_NATIVE", "1")
    generic = torch.full((M * N,), float("nan"), device="cuda")
    cuda_rt.run(ck, {"a": a, "b": b, "c": generic, "M": M, "N": N}, c["meta"], grid=grid)
    torch.cuda.synchronize()
    assert cuda_rt.native_launches == before + 1
    assert torch.equal(native, generic)
