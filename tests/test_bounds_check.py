"""CPU: the bounds-checked lowering (EAS_BOUNDS_CHECK=1).

The reference has no sanitizer for its kernels (its only checker is the structural ``validate_ir``,
ir.py:86-518); a checked lowering stands in for one here.  Every global and threadgroup access
whose mask holds is tested against its buffer first (``eas_inb``), vector paths and grouped dot
loops are off, the extra parameters follow the hidden ones, and every reference kernel compiles
with NVRTC for sm_100a in this mode.  The runtime side (bounds passed per launch, the error record,
IndexError) is covered in tests/test_runtime_fake_lib.py."""

from __future__ import annotations

import ctypes
import re

import pytest

import goldens
from easy_as_b200.codegen.cuda import CHECK_TG_SLOT, ir_to_cuda
from easy_as_b200.runtime import cuda_ext


def lower(cid: str, checked: bool = True):
    return ir_to_cuda(goldens.ir_from_json(goldens.case(cid)["opt"]), checked=checked)


def test_unchecked_lowering_has_no_checks(monkeypatch):
    monkeypatch.delenv("EAS_BOUNDS_CHECK", raising=False)
    lo = ir_to_cuda(goldens.ir_from_json(goldens.case("add_c1")["opt"]))
    assert not lo.checked and "eas_inb" not in lo.src and "eas_err" not in lo.src
    assert all(p.kind != "check" for p in lo.params)


def test_environment_switch_selects_the_checked_lowering(monkeypatch):
    monkeypatch.setenv("EAS_BOUNDS_CHECK", "1")
    assert ir_to_cuda(goldens.ir_from_json(goldens.case("add_c1")["opt"])).checked


def test_every_add_access_is_checked_per_lane():
    """add (BLOCK 256, 4 lanes per thread): 3 buffers x 4 lanes, each guarded after its mask, and no
    float4 accesses."""
    lo = lower("add_c1")
    body = lo.src[lo.src.index("griddepcontrol.wait"):]
    assert body.count("eas_inb(") == 12
    assert "float4" not in body
    for m in re.finditer(r"eas_inb\((\w+\[\d\]), eas_lo_(\w), eas_n_\w, eas_err, (\d+)u\)", body):
        slot, store = divmod(int(m.group(3)), 2)
        assert "abc"[slot] == m.group(2) and store == (m.group(2) == "c")
    names = [p.name for p in lo.params if p.kind == "check"]
    assert names == ["eas_lo_a", "eas_n_a", "eas_lo_b", "eas_n_b", "eas_lo_c", "eas_n_c", "eas_err"]


def test_mask_is_tested_before_bounds():
    """A masked-off lane must not be tested (it would record a false violation): the bounds test
    is the right operand of && after the mask."""
    lo = lower("add_c1")
    for line in lo.src.splitlines():
        if "eas_inb(" in line and "static" not in line:
            assert re.search(r"\(v\d+\[\d\] && eas_inb\(", line), line


def test_threadgroup_accesses_use_their_allocation_size():
    """Threadgroup allocations are checked against their element count, with slots from
    CHECK_TG_SLOT on."""
    lo = lower("matmul_tiled_full")
    sizes = {}
    for inst in goldens.ir_from_json(goldens.case("matmul_tiled_full")["opt"]).insts:
        if inst.op == "alloc_tg":
            sizes[len(sizes)] = int(inst.args[0])
    found = set()
    for m in re.finditer(r"eas_inb\([^;]*?, 0ull, (\d+)ull, eas_err, (\d+)u\)", lo.src):
        slot = int(m.group(2)) // 2 - CHECK_TG_SLOT
        assert sizes[slot] == int(m.group(1))
        found.add(slot)
    assert found == set(sizes)


def test_dot_and_mma_operand_reads_are_checked():
    """dot loops are emitted one per dot (no grouped or vector B loads); each operand read inside
    a dot or mma is guarded."""
    dot = lower("t_many_dot")
    loop = dot.src[dot.src.index("for (uint32_t eas_k = 0;"):]
    assert "eas_inb(eas_ai" in loop and "eas_inb(eas_bi" in loop and "eas_bv" not in loop
    mma = lower("matmul_simdgroup")
    n_mma = sum(i.op == "mma" for i in goldens.ir_from_json(goldens.case("matmul_simdgroup")["opt"]).insts)
    assert n_mma and mma.src.count("eas_pack2((eas_inb(") == 2 * n_mma   # the A and the B pair of each


def _compile(src: str, name: str) -> int:
    lib = cuda_ext.load()
    img, size = ctypes.c_void_p(), ctypes.c_size_t()
    rc = lib.eas_compile(src.encode(), (name + ".cu").encode(), None, 0, ctypes.byref(img), ctypes.byref(size))
    if rc == 0:
        lib.eas_free_host(img)
    return rc


@pytest.mark.parametrize("cid", [c["id"] for c in goldens.cases() if "opt" in c])
def test_checked_reference_kernels_compile_for_sm100a(cid):
    lo = lower(cid)
    assert _compile(lo.src, lo.kernel_name) == 0, cuda_ext.last_error()


def test_checked_fuzz_kernels_compile_and_stay_in_bounds():
    """The differential fuzzer's spmd and thread-mode kernels (tests/fuzz_kernels.py) lower
    checked and compile; the oracle finds no out-of-bounds access in them, so on a GPU their
    checked runs must report none."""
    import fuzz_kernels
    from oracle.interp import execute

    for seed in range(0, 40, 8):
        k, _src = fuzz_kernels.make(seed)
        n = 300 + seed
        args = fuzz_kernels.inputs(seed, n)
        ck = k.compile(*(args[a] for a in ("x", "y", "h", "out", "outi", "outh", "N", "S", "alpha")), BLOCK=64)
        execute(ck.ir, dict(args), grid=(-(-n // 64), 1, 1))
        lo = ir_to_cuda(ck.ir, checked=True)
        assert _compile(lo.src, lo.kernel_name) == 0, cuda_ext.last_error()
    for seed in range(0, 30, 6):
        k, _src, meta = fuzz_kernels.make_thread(seed)
        n = 500 + 11 * seed
        args = fuzz_kernels.thread_inputs(seed, n)
        ck = k.compile(*(args[a] for a in ("x", "y", "out", "N", "S", "alpha")), **meta)
        lo = ir_to_cuda(ck.ir, checked=True)
        assert _compile(lo.src, lo.kernel_name) == 0, cuda_ext.last_error()
