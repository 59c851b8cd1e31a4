"""Structure of the generated CUDA, restating what the reference's MSL-string tests check
(tests/test_spmd_codegen.py, test_f16_codegen.py, test_dot_f16_codegen.py,
test_matmul_tiled.py:103-126, test_mma_codegen.py, test_threadgroup_memory.py:45-75,
test_local_and_lane_id.py:32-39, test_bool_simplify.py, test_fma.py, test_dot_dynamic_k.py:52-59,
test_dot_codegen_unique_vars.py, test_specialize_scalars.py) for the CUDA emitter."""

import re

import numpy as np

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
    assert "for (uint32_t k = 0; k < K; ++k)" in s
    assert "fmaf(" in s


def test_tiled_matmul_groups_dots_with_float4_b_loads(monkeypatch):
    s = src("matmul_tiled_masked")
    assert "const float4 bv = *reinterpret_cast<const float4*>" in s
    assert s.count("const float av =") == 2  # BK steps 1..3 (K=64, BK=16) re-rolled into one loop
    monkeypatch.setenv("EAS_REROLL", "0")
    assert src("matmul_tiled_masked").count("const float av =") == 4  # one grouped k loop per BK step


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
