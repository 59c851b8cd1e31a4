"""Structure of the generated CUDA, restating what the reference's MSL-string tests check
(tests/test_spmd_codegen.py, test_f16_codegen.py, test_dot_f16_codegen.py,
test_matmul_tiled.py:103-126, test_mma_codegen.py, test_threadgroup_memory.py:45-75,
test_local_and_lane_id.py:32-39, test_bool_simplify.py, test_fma.py, test_dot_dynamic_k.py:52-59,
test_dot_codegen_unique_vars.py, test_specialize_scalars.py) for the CUDA emitter."""

import re

import numpy as np
import pytest

import eas
import goldens
from eas import mk
from easy_as_b200.compiler import compile_ir


def src(cid):
    return compile_ir(goldens.ir_from_json(goldens.case(cid)["opt"])).src


def test_spmd_program_is_a_cta_with_vector_accesses():
    s = src("add_c1")
    assert "blockIdx.x + eas_pid_x" in s
    assert "float4" in s and "__launch_bounds__(64, 32)" in s  # 256 lanes = 64 threads x 4


def test_f16_buffers_are_half_bit_patterns():
    @eas.kernel
    def copy16(x, y, N, BLOCK: eas.constexpr):
        offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
        mk.store(y, offs, mk.load(x, offs, offs < N), offs < N)

    h = np.zeros(8, np.float16)
    s = copy16.compile(h, h, 8, BLOCK=128).src
    assert "const eas_h* __restrict__ x" in s and "eas_h* y" in s


def test_dot_reads_f16_as_float_in_a_k_loop():
    s = src("t_gemv_dot")
    assert "for (uint32_t eas_k = 0; eas_k < K; ++eas_k)" in s
    assert "fmaf(" in s


def test_tiled_matmul_groups_dots_with_float4_b_loads(monkeypatch):
    s = src("matmul_tiled_masked")
    assert "const float4 eas_bv = *reinterpret_cast<const float4*>" in s
    assert s.count("const float eas_av =") == 2  # BK steps 1..3 (K=64, BK=16) re-rolled into one loop
    monkeypatch.setenv("EAS_REROLL", "0")
    assert src("matmul_tiled_masked").count("const float eas_av =") == 4  # one grouped k loop per BK step


def test_mma_uses_tensor_core_mma_sync():
    s = src("matmul_simdgroup")
    assert "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32" in s
    assert "eas_mma_f16(" in s


def test_threadgroup_memory_and_barrier_not_under_a_mask():
    s = src("t_tg_copy_masked")
    assert "extern __shared__ __align__(16) unsigned char eas_smem[];" in s
    assert re.search(r"^  __syncthreads\(\);$", s, re.M)
    assert not re.search(r"^\s{3,}__syncthreads", s, re.M)


def test_local_and_lane_ids():
    assert "threadIdx.x" in src("t_local_id")
    assert "threadIdx.x & 31u" in src("t_lane_id")


def test_bool_masks_are_folded_to_logical_and():
    assert "&&" in src("t_bool_chain")


def test_fma_only_where_the_ir_says():
    assert "fmaf(" in src("t_fma_simple")
    s = src("add_c1")
    assert "fmaf(" not in s and "__fadd_rn(" in s  # separately rounded add


def test_runtime_scalars_are_params_constexpr_are_not():
    s = src("add_c1")
    assert "const uint32_t N" in s
    sig = s[s.index("add_kernel("):s.index(") {", s.index("add_kernel("))]
    assert "BLOCK" not in sig


def test_many_dots_share_one_loop_without_redeclaration():
    s = src("t_many_dot")
    assert s.count("uint32_t ai =") == len(re.findall(r"for \(uint32_t k", s))


def test_written_buffers_are_not_const():
    s = src("add_c1")
    assert "const float* __restrict__ a" in s and "float* c" in s and "const float* __restrict__ c" not in s


@eas.kernel
def names_mma_f32(a, b, c, K: eas.constexpr):
    """f32 mk.mma on buffers named a, b and c."""
    _t = mk.tid(0, 32)
    acc = mk.mma_zero()
    for k0 in range(0, K, 8):
        acc = mk.mma(a, k0, K, b, k0 * 8, 8, acc)
    mk.mma_store(c, 0, 8, acc)


@eas.kernel
def names_dot(ai, bi, av, k, t, BLOCK: eas.constexpr):
    """dot on buffers named like the emitter's loop variables, with a scalar named k."""
    r = mk.program_id(0) * BLOCK + mk.tid(0, BLOCK)
    mk.store(av, r, mk.dot(ai, r * k, 1, bi, 0, 1, k), r < t)


@eas.kernel
def names_spmd(d0, d1, i, BLOCK: eas.constexpr):
    """spmd lane loops with a scalar named i."""
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    mk.store(d1, offs, mk.load(d0, offs, offs < i) * 2.0, offs < i)


@eas.kernel
def names_keywords(float4, reinterpret_cast, uint32_t, fmaf, float4_p, BLOCK: eas.constexpr):
    """Names of C++ keywords, types and functions the generated code uses, and one that equals the
    renamed form of another."""
    offs = mk.program_id(0) * BLOCK + mk.arange(0, BLOCK)
    m = offs < uint32_t
    mk.store(reinterpret_cast, offs, mk.fma(mk.load(float4, offs, m), fmaf, mk.load(float4_p, offs, m)), m)


@pytest.mark.parametrize("checked", [False, True])
def test_user_names_do_not_collide_with_generated_locals(checked):
    """Buffers and scalars may be named like the generated kernel's own locals (a, i, k, ai, bi,
    av, t, d0, d1), which carry the reserved eas_ prefix, or like C++ keywords and the types and
    functions the generated code calls, which are renamed: every kernel compiles."""
    import ctypes

    from easy_as_b200.codegen.cuda import ir_to_cuda
    from easy_as_b200.runtime import cuda_ext

    f32 = np.float32
    cases = [
        names_keywords.compile(np.ones(100, f32), np.zeros(100, f32), 100, 2.0, np.ones(100, f32), BLOCK=64),
        names_mma_f32.compile(np.ones(128, f32), np.ones(128, f32), np.zeros(64, f32), K=16),
        names_dot.compile(np.ones(64, f32), np.ones(8, f32), np.zeros(8, f32), 8, 8, BLOCK=32),
        names_spmd.compile(np.ones(100, f32), np.zeros(100, f32), 100, BLOCK=64),
    ]
    lib = cuda_ext.load()
    for ck in cases:
        lo = ir_to_cuda(ck.ir, checked=checked)
        img, size = ctypes.c_void_p(), ctypes.c_size_t()
        rc = lib.eas_compile(lo.src.encode(), (lo.kernel_name + ".cu").encode(), None, 0, ctypes.byref(img),
                             ctypes.byref(size))
        assert rc == 0, cuda_ext.last_error()
        lib.eas_free_host(img)
