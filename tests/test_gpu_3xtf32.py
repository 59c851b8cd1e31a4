"""GPU: the opt-in 3xTF32 mode of proven fp32 matmuls (EAS_FP32_MATMUL=3xtf32).

* ``eas_split_tf32`` is bit-exact against a numpy restatement of the TF32 rounding
  (round to nearest, ties away from zero, on the 13 low mantissa bits);
* ``eas_gemm_tf32`` (tcgen05 kind::tf32) on TF32-exact inputs agrees with float64 to f32
  accumulation error;
* proven fp32 matmul kernels in 3xTF32 mode meet rtol 1e-4 against float64 (the fp32 matmul
  tolerance), on the reference's fixtures and on this repository's tiled variants."""

from __future__ import annotations

import numpy as np
import pytest

import goldens
from easy_as_b200.compiler import compile_ir
from easy_as_b200.runtime import cuda_ext

pytestmark = pytest.mark.gpu


def tf32_rna(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32)
    mag = ((u & np.uint32(0x7FFFFFFF)) + np.uint32(0x1000)) & np.uint32(0xFFFFE000)
    return ((u & np.uint32(0x80000000)) | mag).view(np.float32)


def _split_ref(src: np.ndarray, kp: int, transpose: bool) -> np.ndarray:
    """src [batch][rows][k] (or [batch][k][rows] when transposed) -> [batch][rows][2*kp] = [hi | lo]."""
    s = np.swapaxes(src, 1, 2) if transpose else src
    batch, rows, k = s.shape
    hi = tf32_rna(s)
    lo = tf32_rna(s - hi)
    out = np.zeros((batch, rows, 2 * kp), np.float32)
    out[:, :, :k] = hi
    out[:, :, kp:kp + k] = lo
    return out


@pytest.mark.parametrize("batch,rows,k,transpose", [(1, 37, 19, False), (2, 64, 64, False), (1, 37, 19, True),
                                                     (3, 100, 70, True), (1, 1, 1, True), (1, 1, 1, False),
                                                     (2, 33, 1100, False), (1, 70, 130, True)])
def test_split_bit_exact(cuda_rt, batch, rows, k, transpose):
    import torch

    lib = cuda_ext.load()
    rng = np.random.default_rng(rows * k)
    shape = (batch, k, rows) if transpose else (batch, rows, k)
    src = (rng.standard_normal(shape) * np.exp2(rng.integers(-20, 20, shape))).astype(np.float32)
    if src.size >= 3:
        src.reshape(-1)[:3] = [0.0, -0.0, 1.0 + 2.0 ** -11]      # a tie, rounded away from zero
    kp = -(-k // 32) * 32
    d_src = torch.from_numpy(src).cuda()
    d_dst = torch.full((batch, rows, 2 * kp), float("nan"), device="cuda")
    ld = rows if transpose else k
    cuda_ext.check(lib.eas_split_tf32(d_src.data_ptr(), d_dst.data_ptr(), rows, kp, ld, rows, k, batch, rows * k,
                                      int(transpose), None), "split")
    torch.cuda.synchronize()
    got = d_dst.cpu().numpy()
    want = _split_ref(src, kp, transpose)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 128, 64), (1, 200, 72, 36), (1, 512, 512, 256), (2, 300, 260, 100)])
def test_gemm_3xtf32_segments(cuda_rt, batch, M, N, K):
    """eas_gemm_3xtf32 over [hi | lo] rows equals the three-term product of the parts (float64)."""
    import torch

    lib = cuda_ext.load()
    rng = np.random.default_rng(M * 7 + K)
    a = rng.standard_normal((batch, M, K)).astype(np.float32)
    bt = rng.standard_normal((batch, N, K)).astype(np.float32)
    kp = -(-K // 32) * 32
    a2, b2 = _split_ref(a, kp, False), _split_ref(bt, kp, False)
    da, db = torch.from_numpy(a2).cuda(), torch.from_numpy(b2).cuda()
    dc = torch.full((batch, M, N), float("nan"), device="cuda")
    cuda_ext.check(lib.eas_gemm_3xtf32(da.data_ptr(), db.data_ptr(), dc.data_ptr(), M, N, kp, batch, 2 * kp,
                                       2 * M * kp, 2 * kp, 2 * N * kp, N, M * N, 256 if M > 128 else 128, None),
                   "gemm_3xtf32")
    torch.cuda.synchronize()
    ah, al = a2[..., :kp].astype(np.float64), a2[..., kp:].astype(np.float64)
    bh, bl = b2[..., :kp].astype(np.float64), b2[..., kp:].astype(np.float64)
    ref = sum(np.einsum("bmk,bnk->bmn", x, y) for x, y in ((ah, bh), (ah, bl), (al, bh)))
    err = np.abs(dc.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err <= 1e-5, err


@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 128, 64), (1, 200, 72, 36), (1, 512, 512, 256), (2, 300, 260, 100),
                                         (1, 1, 8, 4)])
def test_gemm_tf32_against_float64(cuda_rt, batch, M, N, K):
    import torch

    lib = cuda_ext.load()
    rng = np.random.default_rng(M + N + K)
    a = tf32_rna(rng.standard_normal((batch, M, K)).astype(np.float32))
    bt = tf32_rna(rng.standard_normal((batch, N, K)).astype(np.float32))   # B K-major: [n][k]
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(bt).cuda()
    dc = torch.full((batch, M, N), float("nan"), device="cuda")
    cuda_ext.check(lib.eas_gemm_tf32(da.data_ptr(), db.data_ptr(), dc.data_ptr(), M, N, K, batch, K, M * K, K, N * K,
                                     N, M * N, 256 if M > 128 else 128, None), "gemm_tf32")
    torch.cuda.synchronize()
    code = __import__("ctypes").c_int()
    cuda_ext.check(lib.eas_gemm_status(0, __import__("ctypes").byref(code)), "status")
    assert code.value == 0
    ref = np.einsum("bmk,bnk->bmn", a.astype(np.float64), bt.astype(np.float64))
    err = np.abs(dc.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err <= 1e-5, err


def _fp64_ref(a, b, M, N, K):
    return a.reshape(M, K).astype(np.float64) @ b.reshape(K, N).astype(np.float64)


def _within_fp32_tolerance(got, ref):
    # rtol 1e-4 of the product's scale (sum |a||b| per output bounds the rounding of any order)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())


@pytest.mark.parametrize("cid,scal,M,N,grid", [
    ("matmul_tiled_full", {}, 64, 128, None),
    ("matmul_tiled_masked", {"PID_M_BASE": 0, "PID_N_BASE": 0}, 300, 260, (5, 19, 1)),
    ("matmul_tiled_masked", {"PID_M_BASE": 0, "PID_N_BASE": 0}, 50, 70, (2, 4, 1)),
    ("t_matmul_tiled_33x65x48", {}, 33, 65, (2, 3, 1)),
])
def test_fixture_matmul_in_3xtf32_mode(cuda_rt, monkeypatch, cid, scal, M, N, grid):
    c = goldens.case(cid)
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    K = c["meta"]["K"]
    if cid == "matmul_tiled_full":
        grid = tuple(c["launch"]["grid"])
    rng = np.random.default_rng(M * N)
    a = rng.standard_normal(M * K).astype(np.float32)
    b = rng.standard_normal(K * N).astype(np.float32)
    got = np.full(M * N, np.nan, np.float32)
    monkeypatch.setenv("EAS_FP32_MATMUL", "3xtf32")
    before = cuda_rt.native_launches
    cuda_rt.run(ck, {"a": a, "b": b, "c": got, "M": M, "N": N, **scal}, c["meta"], sync=True, grid=grid)
    assert cuda_rt.native_launches == before + 1, ck.plan.native.last_reason
    assert ck.plan.native.last_mode == "3xtf32"
    _within_fp32_tolerance(got.reshape(M, N), _fp64_ref(a, b, M, N, K))


def test_tiled_variants_in_3xtf32_mode(cuda_rt, monkeypatch):
    from tiled_variants import VARIANTS, grid, tile_mm, tile_mm_batched

    monkeypatch.setenv("EAS_FP32_MATMUL", "3xtf32")
    rng = np.random.default_rng(5)
    for TM, TN, TK, NT, PAD in VARIANTS:
        M, N, K = 3 * TM + 5, 2 * TN + 3, 3 * TK + 7
        a = rng.standard_normal(M * K).astype(np.float32)
        b = rng.standard_normal(K * N).astype(np.float32)
        out = np.full(M * N, np.nan, np.float32)
        before = cuda_rt.native_launches
        tile_mm(a, b, out, M, N, K=K, TM=TM, TN=TN, TK=TK, NT=NT, PAD=PAD, _grid=grid(M, N, TM, TN))
        assert cuda_rt.native_launches == before + 1
        _within_fp32_tolerance(out.reshape(M, N), _fp64_ref(a, b, M, N, K))
    Z, M, N, K = 3, 70, 90, 40
    a = rng.standard_normal(Z * M * K).astype(np.float32)
    b = rng.standard_normal(Z * K * N).astype(np.float32)
    out = np.full(Z * M * N, np.nan, np.float32)
    tile_mm_batched(a, b, out, M, N, K=K, TM=32, TN=32, TK=16, NT=256, _grid=(3, 3, Z))
    ref = np.einsum("zmk,zkn->zmn", a.reshape(Z, M, K).astype(np.float64), b.reshape(Z, K, N).astype(np.float64))
    _within_fp32_tolerance(out.reshape(Z, M, N), ref)


def test_large_matmul_in_3xtf32_mode_is_far_more_accurate_than_one_tf32_pass(cuda_rt, monkeypatch):
    """Config C3 (the reference's unmasked tiled kernel at M = N = K = 2048): 3xTF32 within 1e-4
    of float64 normwise, and several times closer than a single TF32 product of the same operands.

    What remains (~3e-5 here) is the tensor core's own accumulation: each kind::tf32 MMA adds its
    8 products into D with a rounding biased toward zero, 768 times over K' = 3K."""
    import torch

    c = goldens.case("matmul_tiled_c3_full")
    ck = compile_ir(goldens.ir_from_json(c["opt"]))
    M = N = K = 2048
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(M * K, device="cuda", generator=g)
    b = torch.randn(K * N, device="cuda", generator=g)
    out = torch.empty(M * N, device="cuda")
    monkeypatch.setenv("EAS_FP32_MATMUL", "3xtf32")
    cuda_rt.run(ck, {"a": a, "b": b, "c": out, "M": M, "N": N}, c["meta"], sync=True, grid=(N // 32, M // 32, 1))
    assert ck.plan.native.last_mode == "3xtf32"
    rows = slice(0, 64)
    ref = a.view(M, K)[rows].double() @ b.view(K, N).double()
    err3 = ((out.view(M, N)[rows].double() - ref).abs().max() / ref.abs().max()).item()
    a1 = torch.from_numpy(tf32_rna(a.cpu().numpy())).cuda().view(M, K)[rows].double()
    b1 = torch.from_numpy(tf32_rna(b.cpu().numpy())).cuda().view(K, N).double()
    err1 = ((a1 @ b1 - ref).abs().max() / ref.abs().max()).item()
    assert err3 <= 1e-4 and err3 * 4 < err1, (err3, err1)
